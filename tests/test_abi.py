"""CPU tests of the C ABI: the library loads, exports every symbol the public
headers declare, lays out Fav4Args like the C compiler does, and rejects
invalid arguments exactly as the reference does (src/bshd.hip:27-34) --
all without touching a GPU (validation returns before any CUDA call)."""
import ctypes as C
import math
import re
import subprocess
from pathlib import Path

import pytest

import fav4_bshd as F

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))
INVALID = F.CUDA_ERROR_INVALID_VALUE
A16 = 0x10000  # an aligned dummy address (never dereferenced: validation fails first)


def declared_functions():
    names = []
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:int|size_t)\s+(fav4_\w+)\s*\(", text, flags=re.M)
    return names


def test_headers_declare_the_reference_entry_points():
    names = declared_functions()
    assert "fav4_bshd_forward" in names and "fav4_bshd_select_config" in names
    assert len(names) == len(set(names))


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_declared_symbol(lib, name):
    assert hasattr(lib, name)
    out = subprocess.run(["nm", "-D", "--defined-only", str(F.LIB_PATH)], capture_output=True, text=True).stdout
    assert re.search(rf"\bT {name}$", out, flags=re.M), name


def test_probe_library_loads():
    p = F.load_probe_library()
    for name in ("fav4_probe_tma_load", "fav4_probe_gemm_qk", "fav4_probe_gemm_pv", "fav4_probe_bounded_wait",
                 "fav4_probe_status"):
        assert hasattr(p, name)


def test_args_layout_matches_c_compiler(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "fav4_bshd.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(Fav4Args),'
                   'offsetof(Fav4Args,q),offsetof(Fav4Args,k),offsetof(Fav4Args,v),offsetof(Fav4Args,o),'
                   'offsetof(Fav4Args,lse),offsetof(Fav4Args,batch),offsetof(Fav4Args,heads),'
                   'offsetof(Fav4Args,sq),offsetof(Fav4Args,sk),offsetof(Fav4Args,scale));return 0;}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include", str(src), "-o",
                    str(exe)], check=True)
    got = list(map(int, subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()))
    want = [C.sizeof(F.Args)] + [getattr(F.Args, f).offset for f in
                                 ("q", "k", "v", "o", "lse", "batch", "heads", "sq", "sk", "scale")]
    assert got == want


def make_args(**kw):
    a = dict(q=A16, k=A16 * 2, v=A16 * 3, o=A16 * 4, lse=None, batch=2, heads=8, sq=64, sk=64,
             scale=1 / math.sqrt(128))
    a.update(kw)
    return F.Args(a["q"], a["k"], a["v"], a["o"], a["lse"], a["batch"], a["heads"], a["sq"], a["sk"], a["scale"])


INVALID_CASES = [
    dict(q=None), dict(k=None), dict(v=None), dict(o=None),
    dict(batch=0), dict(heads=0), dict(sq=0), dict(sk=0), dict(batch=-1), dict(sq=-5),
    dict(scale=0.0), dict(scale=-1.0), dict(scale=float("nan")), dict(scale=float("inf")),
    dict(q=A16 + 8), dict(k=A16 + 2), dict(v=A16 + 1), dict(o=A16 + 4),
    dict(batch=2 ** 20, heads=2 ** 12),                  # batch*heads overflows INT_MAX
    dict(heads=2 ** 24 + 1),                              # heads*128 overflows
    dict(heads=64, sq=2 ** 18 + 1),                       # sq*heads*128 overflows
    dict(heads=64, sk=2 ** 18 + 1),                       # sk*heads*128 overflows
]


@pytest.mark.parametrize("kw", INVALID_CASES, ids=[str(c) for c in INVALID_CASES])
def test_forward_rejects_invalid_arguments(lib, kw):
    a = make_args(**kw)
    assert lib.fav4_bshd_forward(C.byref(a), 0, 0, None) == INVALID
    assert lib.fav4_bshd_forward(C.byref(a), 1, 2, None) == INVALID


@pytest.mark.parametrize("causal,config", [(2, 0), (-1, 0), (0, 4), (0, -1), (1, 7)])
def test_forward_rejects_bad_mode_or_config(lib, causal, config):
    a = make_args()
    assert lib.fav4_bshd_forward(C.byref(a), causal, config, None) == INVALID


def test_forward_rejects_null_args(lib):
    assert lib.fav4_bshd_forward(None, 0, 0, None) == INVALID


def test_select_config_auto_rule(lib):
    # reference src/bshd.hip:23-25: sq < 128 -> 1, else 2
    for sq, want in ((1, 1), (127, 1), (128, 2), (4096, 2)):
        a = make_args(sq=sq)
        assert lib.fav4_bshd_select_config(C.byref(a)) == want


@pytest.mark.parametrize("kv", [(-1, 10), (10, 10), (20, 10), (0, 65)])
def test_partial_rejects_bad_kv_range(lib, kv):
    a = make_args(lse=A16 * 5)
    assert lib.fav4_bshd_forward_partial(C.byref(a), 1, 0, kv[0], kv[1], None) == INVALID


def test_partial_requires_lse(lib):
    a = make_args(lse=None)
    assert lib.fav4_bshd_forward_partial(C.byref(a), 0, 0, 0, 64, None) == INVALID
    a = make_args(lse=A16 * 5 + 2)
    assert lib.fav4_bshd_forward_partial(C.byref(a), 0, 0, 0, 64, None) == INVALID


def test_combine_rejects_invalid_arguments(lib):
    o = (C.c_void_p * 2)(A16, A16 * 2)
    lse = (C.c_void_p * 2)(A16 * 3, A16 * 4)
    f = lib.fav4_bshd_combine
    assert f(o, lse, 0, A16 * 5, None, 1, 8, 64, None) == INVALID        # no parts
    assert f(o, lse, 17, A16 * 5, None, 1, 8, 64, None) == INVALID       # too many
    assert f(o, lse, 2, None, None, 1, 8, 64, None) == INVALID           # no output
    assert f(o, lse, 2, A16 * 5 + 8, None, 1, 8, 64, None) == INVALID    # misaligned output
    assert f(o, lse, 2, A16 * 5, None, 0, 8, 64, None) == INVALID        # empty batch
    bad = (C.c_void_p * 2)(A16, None)
    assert f(bad, lse, 2, A16 * 5, None, 1, 8, 64, None) == INVALID      # null part


def _host_case(n_outs=2, lse=(True, False), **kw):
    a = make_args(o=None, **kw)
    outs = (F.HostOut * max(n_outs, 1))()
    for j in range(n_outs):
        outs[j] = F.HostOut(A16 * (6 + j), A16 * 9 if lse[j % len(lse)] else None, j % 2, 0)
    return a, outs


def test_host_workspace_bytes_formula(lib):
    # B=5 cut into 3 chunks -> pieces of 2, 2, 1 batch entries, two staging slots
    a, outs = _host_case(batch=5, heads=8, sq=64, sk=96)
    r256 = lambda n: (n + 255) // 256 * 256  # noqa: E731
    q = r256(2 * 64 * 8 * 256)
    kv = r256(2 * 96 * 8 * 256)
    lse = r256(2 * 8 * 64 * 4)
    slot = q + 2 * kv + 2 * q + lse  # two outputs, only the first with LSE
    assert lib.fav4_bshd_host_workspace_bytes(C.byref(a), outs, 2, 3) == 2 * slot
    # one chunk -> one slot; more chunks than batch entries -> one entry each
    assert lib.fav4_bshd_host_workspace_bytes(C.byref(a), outs, 2, 1) == \
        r256(5 * 64 * 8 * 256) * 3 + 2 * r256(5 * 96 * 8 * 256) + r256(5 * 8 * 64 * 4)
    one = r256(64 * 8 * 256) * 3 + 2 * r256(96 * 8 * 256) + r256(8 * 64 * 4)
    assert lib.fav4_bshd_host_workspace_bytes(C.byref(a), outs, 2, 99) == 2 * one
    assert lib.fav4_bshd_host_workspace_bytes(C.byref(a), outs, 0, 3) == 0
    assert lib.fav4_bshd_host_workspace_bytes(C.byref(a), outs, 9, 3) == 0
    assert lib.fav4_bshd_host_workspace_bytes(C.byref(a), outs, 2, 0) == 0


def test_host_forward_rejects_invalid_arguments(lib):
    a, outs = _host_case()
    need = lib.fav4_bshd_host_workspace_bytes(C.byref(a), outs, 2, 2)
    f = lib.fav4_bshd_forward_host
    ws = A16 * 16
    assert f(C.byref(a), outs, 2, 2, ws, need - 1, None) == INVALID      # workspace too small
    assert f(C.byref(a), outs, 2, 2, ws + 128, need, None) == INVALID    # misaligned workspace
    assert f(C.byref(a), outs, 2, 2, None, need, None) == INVALID        # no workspace
    assert f(C.byref(a), None, 2, 2, ws, need, None) == INVALID          # no outputs
    assert f(C.byref(a), outs, 0, 2, ws, need, None) == INVALID
    for kw in (dict(q=None), dict(k=None), dict(v=None), dict(scale=0.0), dict(sq=0), dict(batch=0)):
        b, o2 = _host_case(**kw)
        assert f(C.byref(b), o2, 2, 2, ws, need, None) == INVALID, kw
    bad = [F.HostOut(None, None, 0, 0), F.HostOut(A16, None, 2, 0), F.HostOut(A16, None, 0, 4)]
    for h in bad:
        o1 = (F.HostOut * 1)(h)
        assert f(C.byref(a), o1, 1, 2, ws, need, None) == INVALID


@pytest.mark.parametrize("kv_heads", [0, -1, 3, 16, 5])
def test_gqa_rejects_bad_kv_heads(lib, kv_heads):
    a = make_args(heads=8)
    assert lib.fav4_bshd_forward_gqa(C.byref(a), kv_heads, 0, 0, None) == INVALID


@pytest.mark.parametrize("kw", INVALID_CASES[:14], ids=[str(c) for c in INVALID_CASES[:14]])
def test_gqa_rejects_invalid_arguments(lib, kw):
    a = make_args(**kw)
    assert lib.fav4_bshd_forward_gqa(C.byref(a), 1, 1, 0, None) == INVALID


def test_splitkv_workspace_bytes(lib):
    a = make_args(batch=2, heads=8, sq=16, sk=4096)
    r256 = lambda n: (n + 255) // 256 * 256  # noqa: E731
    per = r256(2 * 16 * 8 * 256) + r256(2 * 8 * 16 * 4)
    assert lib.fav4_bshd_splitkv_workspace_bytes(C.byref(a), 5) == 5 * per
    assert lib.fav4_bshd_splitkv_workspace_bytes(C.byref(a), 1) == 0
    assert lib.fav4_bshd_splitkv_workspace_bytes(C.byref(a), 0) == 0
    assert lib.fav4_bshd_splitkv_workspace_bytes(C.byref(a), 33) == 0


def test_splitkv_rejects_invalid_arguments(lib):
    a = make_args(batch=1, heads=8, sq=16, sk=4096)
    need = lib.fav4_bshd_splitkv_workspace_bytes(C.byref(a), 4)
    f = lib.fav4_bshd_forward_splitkv
    ws = A16 * 256
    assert f(C.byref(a), 0, 0, 33, ws, need, None) == INVALID
    assert f(C.byref(a), 0, 0, -1, ws, need, None) == INVALID
    assert f(C.byref(a), 0, 0, 4, ws, need - 1, None) == INVALID      # workspace too small
    assert f(C.byref(a), 0, 0, 4, ws + 128, need, None) == INVALID    # misaligned
    assert f(C.byref(a), 0, 0, 4, None, need, None) == INVALID
    assert f(C.byref(a), 2, 0, 4, ws, need, None) == INVALID          # bad mode
    b = make_args(q=None)
    assert f(C.byref(b), 0, 0, 4, ws, need, None) == INVALID


def test_backward_rejects_invalid_arguments(lib):
    def bwd(**kw):
        a = dict(q=A16, k=A16 * 2, v=A16 * 3, o=A16 * 4, dout=A16 * 5, lse=A16 * 6, dq=A16 * 7, dk=A16 * 8,
                 dv=A16 * 9, batch=2, heads=4, sq=64, sk=80, scale=0.1)
        a.update(kw)
        return F.BwdArgs(*(a[n] for n in ("q", "k", "v", "o", "dout", "lse", "dq", "dk", "dv")), a["batch"],
                         a["heads"], a["sq"], a["sk"], a["scale"])
    good = bwd()
    need = lib.fav4_bshd_backward_workspace_bytes(C.byref(good))
    # D and LSE * log2(e) over one padded query tile, then the FP32 dQ accumulator
    assert need == 2 * (2 * 4 * 128 * 4) + 2 * 4 * 128 * 128 * 4
    assert lib.fav4_bshd_backward_workspace_bytes(C.byref(bwd(sq=129))) == 2 * (need - 2 * (2 * 4 * 128 * 4)) + \
        2 * (2 * 2 * 4 * 128 * 4)
    ws = A16 * 256
    for f in (lib.fav4_bshd_backward, lib.fav4_bshd_backward_deterministic):
        for kw in (dict(q=None), dict(dout=None), dict(lse=None), dict(dk=None), dict(batch=0), dict(sk=0),
                   dict(scale=0.0), dict(scale=float("nan")), dict(dq=A16 + 8), dict(lse=A16 + 2),
                   dict(heads=2 ** 24 + 1)):
            assert f(C.byref(bwd(**kw)), 0, ws, need, None) == INVALID, kw
        assert f(C.byref(good), 2, ws, need, None) == INVALID        # bad mode
        assert f(C.byref(good), 0, ws, need - 1, None) == INVALID    # workspace too small
        assert f(C.byref(good), 0, ws + 128, need, None) == INVALID  # misaligned
        assert f(C.byref(good), 0, None, need, None) == INVALID
    g = lib.fav4_bshd_backward_gqa
    for kv, det in ((0, 0), (3, 0), (-2, 1), (8, 0), (2, 2), (2, -1)):
        assert g(C.byref(good), kv, 0, det, ws, need, None) == INVALID, (kv, det)
    assert g(C.byref(bwd(q=None)), 2, 0, 0, ws, need, None) == INVALID
    assert g(None, 2, 0, 0, ws, need, None) == INVALID
    assert g(C.byref(good), 2, 2, 0, ws, need, None) == INVALID     # bad mode


def test_varlen_backward_rejects_invalid_arguments(lib):
    def vb(**kw):
        a = dict(q=A16, k=A16 * 2, v=A16 * 3, o=A16 * 4, dout=A16 * 5, lse=A16 * 6, dq=A16 * 7, dk=A16 * 8,
                 dv=A16 * 9, cu_seqlens_q=A16 * 10, cu_seqlens_k=A16 * 11, batch=3, heads=8, kv_heads=2, max_sq=100,
                 max_sk=150, total_q=200, total_k=300, scale=0.1)
        a.update(kw)
        return F.VarlenBwdArgs(*(a[n] for n in ("q", "k", "v", "o", "dout", "lse", "dq", "dk", "dv", "cu_seqlens_q",
                                                "cu_seqlens_k", "batch", "heads", "kv_heads", "max_sq", "max_sk",
                                                "total_q", "total_k", "scale")))
    good = vb()
    need = lib.fav4_bshd_backward_varlen_workspace_bytes(C.byref(good))
    # D and LSE * log2(e) over one padded query tile per (sequence, head), then the FP32 accumulator
    assert need == 2 * (3 * 8 * 128 * 4) + 3 * 8 * 128 * 128 * 4
    ws = A16 * 256
    f = lib.fav4_bshd_backward_varlen
    for kw in (dict(q=None), dict(dout=None), dict(lse=None), dict(dq=None), dict(cu_seqlens_q=None),
               dict(cu_seqlens_k=None), dict(batch=0), dict(kv_heads=3), dict(kv_heads=0), dict(max_sq=0),
               dict(max_sq=201), dict(max_sk=0), dict(max_sk=301), dict(total_k=0), dict(scale=-1.0),
               dict(scale=float("inf")), dict(dk=A16 * 8 + 8), dict(lse=A16 * 6 + 2), dict(cu_seqlens_k=A16 * 11 + 2)):
        assert lib.fav4_bshd_backward_varlen_workspace_bytes(C.byref(vb(**kw))) == 0, kw
        assert f(C.byref(vb(**kw)), 0, ws, need, None) == INVALID, kw
    assert f(C.byref(good), 2, ws, need, None) == INVALID        # bad mode
    assert f(C.byref(good), 0, ws, need - 1, None) == INVALID    # workspace too small
    assert f(C.byref(good), 0, ws + 128, need, None) == INVALID  # misaligned
    assert f(None, 0, ws, need, None) == INVALID


def test_varlen_rejects_invalid_arguments(lib):
    def va(**kw):
        a = dict(q=A16, k=A16 * 2, v=A16 * 3, o=A16 * 4, lse=None, cu_seqlens_q=A16 * 5, cu_seqlens_k=A16 * 6,
                 batch=3, heads=8, kv_heads=8, max_sq=100, total_q=200, total_k=300, scale=0.1)
        a.update(kw)
        return F.VarlenArgs(*(a[n] for n in ("q", "k", "v", "o", "lse", "cu_seqlens_q", "cu_seqlens_k", "batch",
                                             "heads", "kv_heads", "max_sq", "total_q", "total_k", "scale")))
    f = lib.fav4_bshd_forward_varlen
    for kw in (dict(q=None), dict(o=None), dict(cu_seqlens_q=None), dict(cu_seqlens_k=None), dict(batch=0),
               dict(max_sq=0), dict(max_sq=201), dict(kv_heads=3), dict(kv_heads=0), dict(total_k=0),
               dict(scale=-1.0), dict(cu_seqlens_q=A16 * 5 + 2), dict(lse=A16 * 7 + 1), dict(k=A16 + 8)):
        assert f(C.byref(va(**kw)), 0, 0, None) == INVALID, kw
    assert f(C.byref(va()), 2, 0, None) == INVALID
    assert f(C.byref(va()), 0, 5, None) == INVALID
    assert f(None, 0, 0, None) == INVALID


def test_misaligned_lse_is_rejected_by_every_forward_entry(lib):
    # LSE is stored with 4-byte stores; a pointer that is not 4-byte aligned
    # would fault on the GPU, so each entry refuses it before any CUDA call.
    for off in (1, 2, 3):
        a = make_args(batch=1, heads=8, sq=16, sk=4096, lse=A16 * 5 + off)
        ws = A16 * 256
        need = lib.fav4_bshd_splitkv_workspace_bytes(C.byref(a), 4)
        assert lib.fav4_bshd_forward(C.byref(a), 0, 0, None) == INVALID
        assert lib.fav4_bshd_forward(C.byref(a), 1, 2, None) == INVALID
        assert lib.fav4_bshd_forward_gqa(C.byref(a), 2, 0, 0, None) == INVALID
        assert lib.fav4_bshd_forward_partial(C.byref(a), 0, 0, 0, 64, None) == INVALID
        assert lib.fav4_bshd_forward_splitkv(C.byref(a), 0, 0, 4, ws, need, None) == INVALID
        assert lib.fav4_bshd_forward_partial_splitkv(C.byref(a), 0, 0, 0, 4096, 4, ws, need, None) == INVALID
        assert lib.fav4_bshd_forward_splitkv_static(C.byref(a), 1, 0, 4, None) == INVALID
        assert lib.fav4_bshd_splitkv_splits(C.byref(a), 0, 0) == -1
        o = (C.c_void_p * 2)(A16, A16 * 2)
        lse = (C.c_void_p * 2)(A16 * 3, A16 * 4)
        assert lib.fav4_bshd_combine(o, lse, 2, A16 * 5, C.c_void_p(A16 * 6 + off), 1, 8, 64, None) == INVALID

"""Python host side of the B200 BF16 attention-forward library.

Mirrors the reference's ctypes harness interface (benchmarks/bshd.py:18-20 for
the ``Args`` structure, :56-74 for ``Runner.call``): the same struct layout,
the same argument checks, the same error behaviour (a nonzero status raises
RuntimeError). Everything runs through the C ABI in include/fav4_bshd.h,
implemented by build/libfav4_bshd.so; there is no other code path, so a
missing library is an error, never a fallback.
"""
from __future__ import annotations

import ctypes as C
import math
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]  # the flash-attention-v4-rocm_b200 folder
BUILD_DIR = PKG_ROOT / "build"
LIB_PATH = BUILD_DIR / "libfav4_bshd.so"
PROBE_LIB_PATH = BUILD_DIR / "libfav4_probe.so"
HEAD_DIM = 128
CUDA_ERROR_INVALID_VALUE = 1


class Args(C.Structure):
    """Fav4Args (include/fav4_bshd.h), field for field as benchmarks/bshd.py:18-20."""

    _fields_ = [(n, C.c_void_p) for n in ("q", "k", "v", "o", "lse")] + [
        (n, C.c_int) for n in ("batch", "heads", "sq", "sk")] + [("scale", C.c_float)]


class BwdArgs(C.Structure):
    """Fav4BwdArgs (include/fav4_bshd.h): arguments of fav4_bshd_backward."""

    _fields_ = [(n, C.c_void_p) for n in ("q", "k", "v", "o", "dout", "lse", "dq", "dk", "dv")] + [
        (n, C.c_int) for n in ("batch", "heads", "sq", "sk")] + [("scale", C.c_float)]


class VarlenArgs(C.Structure):
    """Fav4VarlenArgs (include/fav4_bshd.h): packed variable-length sequences."""

    _fields_ = [(n, C.c_void_p) for n in ("q", "k", "v", "o", "lse", "cu_seqlens_q", "cu_seqlens_k")] + [
        (n, C.c_int) for n in ("batch", "heads", "kv_heads", "max_sq", "total_q", "total_k")] + [("scale", C.c_float)]


class VarlenBwdArgs(C.Structure):
    """Fav4VarlenBwdArgs (include/fav4_bshd.h): backward of packed sequences."""

    _fields_ = [(n, C.c_void_p) for n in ("q", "k", "v", "o", "dout", "lse", "dq", "dk", "dv", "cu_seqlens_q",
                                          "cu_seqlens_k")] + [
        (n, C.c_int) for n in ("batch", "heads", "kv_heads", "max_sq", "max_sk", "total_q", "total_k")] + [
        ("scale", C.c_float)]


class HostOut(C.Structure):
    """Fav4HostOut (include/fav4_bshd.h): one output of fav4_bshd_forward_host."""

    _fields_ = [("o", C.c_void_p), ("lse", C.c_void_p), ("causal", C.c_int), ("config", C.c_int)]


_LIB = None
_PROBE = None


def _bind(lib):
    lib.fav4_bshd_forward.argtypes = [C.POINTER(Args), C.c_int, C.c_int, C.c_void_p]
    lib.fav4_bshd_forward.restype = C.c_int
    lib.fav4_bshd_forward_wide.argtypes = [C.POINTER(Args), C.c_void_p]
    lib.fav4_bshd_forward_wide.restype = C.c_int
    lib.fav4_bshd_select_config.argtypes = [C.POINTER(Args)]
    lib.fav4_bshd_select_config.restype = C.c_int
    lib.fav4_bshd_forward_splitkv.argtypes = [C.POINTER(Args), C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                              C.c_void_p]
    lib.fav4_bshd_forward_splitkv.restype = C.c_int
    lib.fav4_bshd_forward_partial_splitkv.argtypes = [C.POINTER(Args), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                      C.c_void_p, C.c_size_t, C.c_void_p]
    lib.fav4_bshd_forward_partial_splitkv.restype = C.c_int
    lib.fav4_bshd_splitkv_workspace_bytes.argtypes = [C.POINTER(Args), C.c_int]
    lib.fav4_bshd_splitkv_workspace_bytes.restype = C.c_size_t
    lib.fav4_bshd_splitkv_splits.argtypes = [C.POINTER(Args), C.c_int, C.c_int]
    lib.fav4_bshd_splitkv_splits.restype = C.c_int
    lib.fav4_bshd_forward_gqa.argtypes = [C.POINTER(Args), C.c_int, C.c_int, C.c_int, C.c_void_p]
    lib.fav4_bshd_forward_gqa.restype = C.c_int
    lib.fav4_bshd_forward_partial.argtypes = [C.POINTER(Args), C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
    lib.fav4_bshd_forward_partial.restype = C.c_int
    lib.fav4_bshd_combine.argtypes = [C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_int, C.c_void_p,
                                      C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
    lib.fav4_bshd_combine.restype = C.c_int
    lib.fav4_bshd_forward_splitkv_static.argtypes = [C.POINTER(Args), C.c_int, C.c_int, C.c_int, C.c_void_p]
    lib.fav4_bshd_forward_splitkv_static.restype = C.c_int
    lib.fav4_bshd_host_workspace_bytes.argtypes = [C.POINTER(Args), C.POINTER(HostOut), C.c_int, C.c_int]
    lib.fav4_bshd_host_workspace_bytes.restype = C.c_size_t
    lib.fav4_bshd_forward_host.argtypes = [C.POINTER(Args), C.POINTER(HostOut), C.c_int, C.c_int, C.c_void_p,
                                           C.c_size_t, C.c_void_p]
    lib.fav4_bshd_forward_host.restype = C.c_int
    lib.fav4_bshd_backward_workspace_bytes.argtypes = [C.POINTER(BwdArgs)]
    lib.fav4_bshd_backward_workspace_bytes.restype = C.c_size_t
    lib.fav4_bshd_backward.argtypes = [C.POINTER(BwdArgs), C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]
    lib.fav4_bshd_backward.restype = C.c_int
    lib.fav4_bshd_backward_deterministic.argtypes = [C.POINTER(BwdArgs), C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]
    lib.fav4_bshd_backward_deterministic.restype = C.c_int
    lib.fav4_bshd_backward_gqa.argtypes = [C.POINTER(BwdArgs), C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                           C.c_void_p]
    lib.fav4_bshd_backward_gqa.restype = C.c_int
    lib.fav4_bshd_backward_varlen_workspace_bytes.argtypes = [C.POINTER(VarlenBwdArgs)]
    lib.fav4_bshd_backward_varlen_workspace_bytes.restype = C.c_size_t
    lib.fav4_bshd_backward_varlen.argtypes = [C.POINTER(VarlenBwdArgs), C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]
    lib.fav4_bshd_backward_varlen.restype = C.c_int
    lib.fav4_bshd_forward_varlen.argtypes = [C.POINTER(VarlenArgs), C.c_int, C.c_int, C.c_void_p]
    lib.fav4_bshd_forward_varlen.restype = C.c_int
    lib.fav4_bshd_pipeline_status.argtypes = [C.c_int]
    lib.fav4_bshd_pipeline_status.restype = C.c_int
    return lib


def load_library(path: Path | str | None = None):
    """Load (once) the CUDA library. Raises if it has not been built."""
    global _LIB
    if _LIB is None or path is not None:
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(f"{p} is missing: build it with `python -m fav4_bshd.build` "
                               f"(or __graft_entry__.build()); there is no CPU fallback")
        lib = _bind(C.CDLL(str(p)))
        if path is not None:
            return lib
        _LIB = lib
    return _LIB


def load_probe_library():
    """The test-only probe library (TMA / UMMA / bounded-wait probes)."""
    global _PROBE
    if _PROBE is None:
        if not PROBE_LIB_PATH.exists():
            raise RuntimeError(f"{PROBE_LIB_PATH} is missing: build it with `python -m fav4_bshd.build`")
        lib = C.CDLL(str(PROBE_LIB_PATH))
        lib.fav4_probe_tma_load.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
        lib.fav4_probe_gemm_qk.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        lib.fav4_probe_gemm_pv.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        lib.fav4_probe_bounded_wait.argtypes = [C.c_int, C.c_void_p, C.c_void_p]
        lib.fav4_probe_status.argtypes = [C.c_int]
        for f in ("fav4_probe_tma_load", "fav4_probe_gemm_qk", "fav4_probe_gemm_pv", "fav4_probe_bounded_wait",
                  "fav4_probe_status"):
            getattr(lib, f).restype = C.c_int
        _PROBE = lib
    return _PROBE


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(stream=None):
    import torch
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _check_bshd(q, k, v, o, lse, kv_heads=None):
    import torch
    assert all(x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous() for x in (q, k, v, o))
    b, sq, h, d = q.shape
    hk = h if kv_heads is None else kv_heads
    assert d == HEAD_DIM and k.shape == v.shape and k.shape[0] == b and k.shape[2:] == (hk, d) and o.shape == q.shape
    assert lse is None or (lse.shape == (b, h, sq) and lse.is_contiguous() and lse.dtype == torch.float32)
    return b, sq, h


class Runner:
    """The reference harness's Runner (benchmarks/bshd.py:56-74), bound to this library."""

    def __init__(self, lib=None):
        self.lib = lib if lib is not None else load_library()

    def args(self, q, k, v, o, lse, scale=None):
        b, sq, h = _check_bshd(q, k, v, o, lse)
        scale = 1 / math.sqrt(HEAD_DIM) if scale is None else scale
        return Args(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), b, h, sq, k.shape[1], scale)

    def call(self, q, k, v, o, lse, causal, config=0, scale=None, stream=None):
        a = self.args(q, k, v, o, lse, scale)
        status = self.lib.fav4_bshd_forward(C.byref(a), int(causal), config, _stream(stream))
        if status:
            raise RuntimeError(f"config {config}: CUDA status {status}")

    def call_wide(self, q, k, v, o, lse, scale=None, stream=None):
        """Dense forward through the wide-step kernel (fav4_bshd_forward_wide)."""
        a = self.args(q, k, v, o, lse, scale)
        status = self.lib.fav4_bshd_forward_wide(C.byref(a), _stream(stream))
        if status:
            raise RuntimeError(f"wide: CUDA status {status}")

    def call_splitkv(self, q, k, v, o, lse, causal, config=0, splits=0, scale=None, stream=None, workspace=None):
        """Split-KV forward in one launch (fav4_bshd_forward_splitkv), for few
        query tiles against many keys. splits=0 picks the number for this GPU.
        The workspace is allocated with torch (kept for the next call) unless
        one is given. Returns the number of splits used."""
        import torch
        a = self.args(q, k, v, o, lse, scale)
        if splits == 0:
            splits = self.lib.fav4_bshd_splitkv_splits(C.byref(a), int(causal), config)
            if splits < 1:
                raise RuntimeError("splitkv: invalid arguments")
        need = self.lib.fav4_bshd_splitkv_workspace_bytes(C.byref(a), splits)
        if workspace is None and need > 0:
            ws = getattr(self, "_split_ws", None)
            if ws is None or ws.numel() < need or ws.device != q.device:
                ws = self._split_ws = torch.empty(need, dtype=torch.uint8, device=q.device)
            workspace = ws
        ptr, size = (workspace.data_ptr(), workspace.numel()) if workspace is not None else (None, 0)
        status = self.lib.fav4_bshd_forward_splitkv(C.byref(a), int(causal), config, splits, ptr, size,
                                                    _stream(stream))
        if status:
            raise RuntimeError(f"splitkv {splits} splits, config {config}: CUDA status {status}")
        return splits

    def _split_workspace(self, a, splits, device):
        import torch
        need = self.lib.fav4_bshd_splitkv_workspace_bytes(C.byref(a), splits)
        if need == 0:
            return None, 0
        ws = getattr(self, "_split_ws", None)
        if ws is None or ws.numel() < need or ws.device != device:
            ws = self._split_ws = torch.empty(need, dtype=torch.uint8, device=device)
        return ws.data_ptr(), ws.numel()

    def call_partial_splitkv(self, q, k, v, o, lse, causal, kv_begin, kv_end, config=0, splits=1, scale=None,
                             stream=None):
        """fav4_bshd_forward_partial over keys [kv_begin, kv_end) with the
        one-launch split (fav4_bshd_forward_partial_splitkv)."""
        a = self.args(q, k, v, o, lse, scale)
        ptr, size = self._split_workspace(a, splits, q.device)
        status = self.lib.fav4_bshd_forward_partial_splitkv(C.byref(a), int(causal), config, kv_begin, kv_end,
                                                            splits, ptr, size, _stream(stream))
        if status:
            raise RuntimeError(f"partial splitkv [{kv_begin},{kv_end}) x{splits}: CUDA status {status}")

    def call_gqa(self, q, k, v, o, lse, causal, config=0, scale=None, stream=None):
        """Grouped-query attention: k and v have H_kv heads, H_kv dividing q's
        heads (fav4_bshd_forward_gqa)."""
        hk = k.shape[2]
        b, sq, h = _check_bshd(q, k, v, o, lse, kv_heads=hk)
        scale = 1 / math.sqrt(HEAD_DIM) if scale is None else scale
        a = Args(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse), b, h, sq, k.shape[1], scale)
        status = self.lib.fav4_bshd_forward_gqa(C.byref(a), hk, int(causal), config, _stream(stream))
        if status:
            raise RuntimeError(f"gqa kv_heads {hk} config {config}: CUDA status {status}")

    def call_partial(self, q, k, v, o, lse, causal, kv_begin, kv_end, config=0, scale=None, stream=None):
        a = self.args(q, k, v, o, lse, scale)
        status = self.lib.fav4_bshd_forward_partial(C.byref(a), int(causal), config, kv_begin, kv_end,
                                                    _stream(stream))
        if status:
            raise RuntimeError(f"partial [{kv_begin},{kv_end}) config {config}: CUDA status {status}")

    def combine(self, o_parts, lse_parts, o, lse=None, stream=None):
        import torch
        n = len(o_parts)
        assert n == len(lse_parts) and n >= 1
        b, sq, h, d = o.shape
        assert o.dtype == torch.bfloat16 and o.is_contiguous() and d == HEAD_DIM
        for op, lp in zip(o_parts, lse_parts):
            assert op.shape == o.shape and op.dtype == torch.bfloat16 and op.is_contiguous()
            assert lp.shape == (b, h, sq) and lp.dtype == torch.float32 and lp.is_contiguous()
        optrs = (C.c_void_p * n)(*[x.data_ptr() for x in o_parts])
        lptrs = (C.c_void_p * n)(*[x.data_ptr() for x in lse_parts])
        status = self.lib.fav4_bshd_combine(optrs, lptrs, n, o.data_ptr(), _ptr(lse), b, h, sq, _stream(stream))
        if status:
            raise RuntimeError(f"combine of {n} parts: CUDA status {status}")

    def forward_host(self, q, k, v, outs, chunks=8, scale=None, stream=None, workspace=None):
        """Forwards of host-resident (page-locked) Q/K/V through
        fav4_bshd_forward_host: one upload, one output per (o, lse, causal,
        config) in `outs` (o, lse: host tensors; lse may be None), copies and
        kernels overlapped over `chunks` batch pieces. Ordered on `stream`;
        the host outputs are complete once that stream is synchronised. The
        device workspace is allocated with torch (and kept for the next call
        of the same shape) unless one is given."""
        import torch
        assert all(x.dtype == torch.bfloat16 and not x.is_cuda and x.is_contiguous() for x in (q, k, v))
        b, sq, h, d = q.shape
        assert d == HEAD_DIM and k.shape == v.shape and k.shape[0] == b and k.shape[2:] == (h, d)
        ho = (HostOut * len(outs))()
        for j, (o, lse, causal, config) in enumerate(outs):
            assert o.shape == q.shape and o.dtype == torch.bfloat16 and not o.is_cuda and o.is_contiguous()
            assert lse is None or (lse.shape == (b, h, sq) and lse.dtype == torch.float32 and not lse.is_cuda)
            ho[j] = HostOut(o.data_ptr(), _ptr(lse), int(causal), int(config))
        scale = 1 / math.sqrt(HEAD_DIM) if scale is None else scale
        a = Args(q.data_ptr(), k.data_ptr(), v.data_ptr(), None, None, b, h, sq, k.shape[1], scale)
        need = self.lib.fav4_bshd_host_workspace_bytes(C.byref(a), ho, len(outs), chunks)
        if need == 0:
            raise RuntimeError("forward_host: invalid arguments")
        if workspace is None:
            ws = getattr(self, "_host_ws", None)
            if ws is None or ws.numel() < need or ws.device != torch.device("cuda", torch.cuda.current_device()):
                ws = self._host_ws = torch.empty(need, dtype=torch.uint8, device="cuda")
            workspace = ws
        assert workspace.is_cuda and workspace.numel() >= need
        status = self.lib.fav4_bshd_forward_host(C.byref(a), ho, len(outs), chunks, workspace.data_ptr(),
                                                 workspace.numel(), _stream(stream))
        if status:
            raise RuntimeError(f"forward_host: CUDA status {status}")

    def call_varlen(self, q, k, v, o, lse, cu_q, cu_k, max_sq, causal, config=0, scale=None, stream=None):
        """Packed sequences (fav4_bshd_forward_varlen): q, o [total_q, H, 128];
        k, v [total_k, H_kv, 128]; cu_q, cu_k int32 CUDA [batch + 1]; lse
        optional FP32 [H, total_q]."""
        import torch
        for x in (q, k, v, o):
            assert x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous() and x.dim() == 3
        assert cu_q.dtype == cu_k.dtype == torch.int32 and cu_q.is_cuda and cu_k.is_cuda
        assert cu_q.numel() == cu_k.numel() >= 2 and o.shape == q.shape and k.shape == v.shape
        tq, h, _ = q.shape
        tk, hk, _ = k.shape
        assert lse is None or (lse.shape == (h, tq) and lse.dtype == torch.float32 and lse.is_contiguous())
        scale = 1 / math.sqrt(HEAD_DIM) if scale is None else scale
        a = VarlenArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), _ptr(lse), cu_q.data_ptr(),
                       cu_k.data_ptr(), cu_q.numel() - 1, h, hk, max_sq, tq, tk, scale)
        status = self.lib.fav4_bshd_forward_varlen(C.byref(a), int(causal), config, _stream(stream))
        if status:
            raise RuntimeError(f"varlen config {config}: CUDA status {status}")

    def backward_varlen(self, q, k, v, o, dout, lse, dq, dk, dv, cu_q, cu_k, max_sq, max_sk, causal, scale=None,
                        stream=None):
        """Gradients of call_varlen (fav4_bshd_backward_varlen): q, o, dout, dq
        [total_q, H, 128]; k, v, dk, dv [total_k, H_kv, 128]; lse the forward's FP32
        [H, total_q]; cu_q, cu_k int32 CUDA [batch + 1]; max_sq / max_sk bound the
        sequence lengths. The workspace is allocated with torch and kept."""
        import torch
        for x in (q, k, v, o, dout, dq, dk, dv):
            assert x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous() and x.dim() == 3
        assert cu_q.dtype == cu_k.dtype == torch.int32 and cu_q.is_cuda and cu_k.is_cuda
        assert cu_q.numel() == cu_k.numel() >= 2
        assert o.shape == dout.shape == dq.shape == q.shape and k.shape == v.shape == dk.shape == dv.shape
        tq, h, _ = q.shape
        tk, hk, _ = k.shape
        assert lse.shape == (h, tq) and lse.dtype == torch.float32 and lse.is_contiguous()
        scale = 1 / math.sqrt(HEAD_DIM) if scale is None else scale
        a = VarlenBwdArgs(*(x.data_ptr() for x in (q, k, v, o, dout, lse, dq, dk, dv, cu_q, cu_k)),
                          cu_q.numel() - 1, h, hk, max_sq, max_sk, tq, tk, scale)
        need = self.lib.fav4_bshd_backward_varlen_workspace_bytes(C.byref(a))
        if need == 0:
            raise RuntimeError("backward_varlen: invalid arguments")
        ws = getattr(self, "_bwd_ws", None)
        if ws is None or ws.numel() < need or ws.device != q.device:
            ws = self._bwd_ws = torch.empty(need, dtype=torch.uint8, device=q.device)
        status = self.lib.fav4_bshd_backward_varlen(C.byref(a), int(causal), ws.data_ptr(), ws.numel(),
                                                    _stream(stream))
        if status:
            raise RuntimeError(f"backward_varlen: CUDA status {status}")

    def backward(self, q, k, v, o, dout, lse, dq, dk, dv, causal, scale=None, stream=None, deterministic=False):
        """dQ, dK, dV through fav4_bshd_backward, or fav4_bshd_backward_deterministic
        (all BF16 BSHD CUDA tensors, lse the forward's FP32 [B, H, Sq]). k, v, dk,
        dv may have fewer heads than q, a divisor of q's (grouped-query attention,
        through fav4_bshd_backward_gqa). The workspace is allocated with torch and
        kept for the next call."""
        import torch
        for x in (q, k, v, o, dout, dq, dk, dv):
            assert x.dtype == torch.bfloat16 and x.is_cuda and x.is_contiguous()
        b, sq, h, d = q.shape
        hk = k.shape[2]
        assert d == HEAD_DIM and k.shape == v.shape == dk.shape == dv.shape and k.shape[0] == b and h % hk == 0
        assert o.shape == dout.shape == dq.shape == q.shape
        assert lse.shape == (b, h, sq) and lse.dtype == torch.float32 and lse.is_contiguous()
        scale = 1 / math.sqrt(HEAD_DIM) if scale is None else scale
        a = BwdArgs(*(x.data_ptr() for x in (q, k, v, o, dout, lse, dq, dk, dv)), b, h, sq, k.shape[1], scale)
        need = self.lib.fav4_bshd_backward_workspace_bytes(C.byref(a))
        ws = getattr(self, "_bwd_ws", None)
        if ws is None or ws.numel() < need or ws.device != q.device:
            ws = self._bwd_ws = torch.empty(need, dtype=torch.uint8, device=q.device)
        if hk != h:
            status = self.lib.fav4_bshd_backward_gqa(C.byref(a), hk, int(causal), int(bool(deterministic)),
                                                     ws.data_ptr(), ws.numel(), _stream(stream))
        else:
            fn = self.lib.fav4_bshd_backward_deterministic if deterministic else self.lib.fav4_bshd_backward
            status = fn(C.byref(a), int(causal), ws.data_ptr(), ws.numel(), _stream(stream))
        if status:
            raise RuntimeError(f"backward: CUDA status {status}")

    def select_config(self, q, k, v, o, lse=None):
        a = self.args(q, k, v, o, lse)
        return self.lib.fav4_bshd_select_config(C.byref(a))

    def pipeline_status(self, clear=True):
        return self.lib.fav4_bshd_pipeline_status(1 if clear else 0)


def forward(q, k, v, causal=False, config=0, scale=None, return_lse=False, out=None):
    """Allocate O (and LSE) with torch and run fav4_bshd_forward on the current stream."""
    import torch
    o = torch.empty_like(q) if out is None else out
    lse = torch.empty((q.shape[0], q.shape[2], q.shape[1]), device=q.device, dtype=torch.float32) \
        if return_lse else None
    Runner().call(q, k, v, o, lse, causal, config, scale)
    return (o, lse) if return_lse else o


__all__ = ["Args", "BwdArgs", "VarlenArgs", "HostOut", "Runner", "forward", "load_library", "load_probe_library", "LIB_PATH", "PROBE_LIB_PATH",
           "HEAD_DIM", "CUDA_ERROR_INVALID_VALUE"]

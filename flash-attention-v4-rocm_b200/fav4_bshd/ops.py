"""PyTorch operator for the attention forward: ``torch.ops.fav4.bshd_forward``.

The reference's callers build the ``Fav4Args`` structure by hand for every
call (benchmarks/bshd.py:64-74). This module registers the C ABI as a PyTorch
custom operator instead, so a caller passes tensors and PyTorch handles the
output allocation, the current stream and tracing:

    o, lse = torch.ops.fav4.bshd_forward(q, k, v, causal, config, scale, return_lse)

* q, k, v: CUDA BF16 ``[B, S, H, 128]``, contiguous (the reference contract,
  include/fav4_bshd.h:12-15); k and v share their shape. k and v may have
  fewer heads than q, a divisor of q's (grouped-query attention, through
  fav4_bshd_forward_gqa).
* causal: top-left causal mask. config: 0 (Auto) to 3. scale: softmax scale,
  or a non-positive value for 1/sqrt(128).
* Returns O (BF16, q's shape) and LSE (FP32 ``[B, H, Sq]``, natural log), or
  an empty LSE tensor when ``return_lse`` is False.

``torch.ops.fav4.varlen_forward`` (``varlen_attention()``) is the same for
packed sequences ``[total, H, 128]`` with int32 ``cu_seqlens`` offsets,
differentiable through ``fav4_bshd_backward_varlen``.

The CUDA kernel runs through ``fav4_bshd_forward`` on the current stream, so
the operator can be captured in a CUDA graph. A fake (meta) implementation
gives shapes to FakeTensor tracing and ``torch.compile`` graphs, so the op
composes with both. Gradients of O with respect to q, k, v come from
``fav4_bshd_backward`` (``fav4_bshd_backward_gqa`` for grouped-query
attention: dK and dV of a K/V head sum over its query heads); they need the
LSE, so call the op with ``return_lse=True`` (``attention()`` does). A gradient
through the LSE output is not implemented and raises.
"""
from __future__ import annotations

import math

import torch

from . import HEAD_DIM, Runner

_RUNNER: Runner | None = None


def _runner() -> Runner:
    global _RUNNER
    if _RUNNER is None:
        _RUNNER = Runner()
    return _RUNNER


def _check(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, config: int) -> None:
    torch._check(q.dim() == 4 and q.shape[-1] == HEAD_DIM, lambda: f"q must be [B, S, H, {HEAD_DIM}], got {q.shape}")
    torch._check(k.shape == v.shape, lambda: f"k and v shapes differ: {k.shape} vs {v.shape}")
    torch._check(k.dim() == 4 and k.shape[0] == q.shape[0] and k.shape[3] == HEAD_DIM and k.shape[2] >= 1
                 and q.shape[2] % k.shape[2] == 0,
                 lambda: f"k must be [B, Sk, H_kv, {HEAD_DIM}] with q's B and H_kv dividing q's heads, got {k.shape}")
    torch._check(all(x.dtype == torch.bfloat16 for x in (q, k, v)), lambda: "q, k, v must be bfloat16")
    torch._check(0 <= config <= 3, lambda: f"config must be 0..3, got {config}")


@torch.library.custom_op("fav4::bshd_forward", mutates_args=(), device_types="cuda")
def bshd_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, config: int, scale: float,
                 return_lse: bool) -> tuple[torch.Tensor, torch.Tensor]:
    _check(q, k, v, config)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    o = torch.empty_like(q)
    b, sq, h, _ = q.shape
    lse = torch.empty((b, h, sq) if return_lse else (0,), device=q.device, dtype=torch.float32)
    sc = 1 / math.sqrt(HEAD_DIM) if scale <= 0 else scale
    with torch.cuda.device(q.device):
        if k.shape[2] == h:
            _runner().call(q, k, v, o, lse if return_lse else None, causal, config, sc)
        else:
            _runner().call_gqa(q, k, v, o, lse if return_lse else None, causal, config, sc)
    return o, lse


@bshd_forward.register_fake
def _(q, k, v, causal, config, scale, return_lse):
    _check(q, k, v, config)
    b, sq, h, _ = q.shape
    o = torch.empty_like(q, memory_format=torch.contiguous_format)
    lse = q.new_empty((b, h, sq) if return_lse else (0,), dtype=torch.float32)
    return o, lse


def _setup_context(ctx, inputs, output):
    q, k, v, causal, config, scale, return_lse = inputs
    o, lse = output
    ctx.save_for_backward(q, k, v, o, lse)
    ctx.causal, ctx.has_lse = causal, return_lse
    ctx.scale = 1 / math.sqrt(HEAD_DIM) if scale <= 0 else scale
    ctx.set_materialize_grads(False)


def _backward(ctx, grad_o, grad_lse):
    q, k, v, o, lse = ctx.saved_tensors
    if grad_lse is not None:
        raise NotImplementedError("fav4::bshd_forward: the gradient through the LSE output is not implemented")
    if not ctx.has_lse:
        raise RuntimeError("fav4::bshd_forward: gradients need return_lse=True (fav4_bshd.ops.attention does this)")
    if grad_o is None:
        return None, None, None, None, None, None, None
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    with torch.cuda.device(q.device):
        _runner().backward(q.contiguous(), k.contiguous(), v.contiguous(), o, grad_o.contiguous(), lse, dq, dk, dv,
                           ctx.causal, ctx.scale)
    return dq, dk, dv, None, None, None, None


bshd_forward.register_autograd(_backward, setup_context=_setup_context)


def _check_varlen(q, k, v, cu_q, cu_k, max_sq, max_sk):
    torch._check(q.dim() == 3 and q.shape[-1] == HEAD_DIM, lambda: f"q must be [total_q, H, {HEAD_DIM}], got {q.shape}")
    torch._check(k.shape == v.shape and k.dim() == 3 and k.shape[-1] == HEAD_DIM and k.shape[1] >= 1
                 and q.shape[1] % k.shape[1] == 0,
                 lambda: f"k, v must be [total_k, H_kv, {HEAD_DIM}] with H_kv dividing q's heads, got {k.shape}")
    torch._check(all(x.dtype == torch.bfloat16 for x in (q, k, v)), lambda: "q, k, v must be bfloat16")
    torch._check(cu_q.dtype == torch.int32 and cu_k.dtype == torch.int32 and cu_q.dim() == 1
                 and cu_q.shape == cu_k.shape and cu_q.shape[0] >= 2,
                 lambda: "cu_seqlens_q / cu_seqlens_k must be int32 [batch + 1]")
    torch._check(1 <= max_sq <= q.shape[0] and 1 <= max_sk <= k.shape[0],
                 lambda: f"max_sq / max_sk must be in [1, total], got {max_sq}, {max_sk}")


@torch.library.custom_op("fav4::varlen_forward", mutates_args=(), device_types="cuda")
def varlen_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                   cu_seqlens_k: torch.Tensor, max_sq: int, max_sk: int, causal: bool,
                   scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Packed sequences (fav4_bshd_forward_varlen): q [total_q, H, 128], k, v
    [total_k, H_kv, 128], device int32 offsets [batch + 1]. Returns O (q's shape)
    and LSE (FP32 [H, total_q]). max_sq / max_sk bound every sequence's length."""
    _check_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_sq, max_sk)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    o = torch.empty_like(q)
    lse = torch.empty((q.shape[1], q.shape[0]), device=q.device, dtype=torch.float32)
    sc = 1 / math.sqrt(HEAD_DIM) if scale <= 0 else scale
    with torch.cuda.device(q.device):
        _runner().call_varlen(q, k, v, o, lse, cu_seqlens_q.contiguous(), cu_seqlens_k.contiguous(), max_sq, causal,
                              0, sc)
    return o, lse


@varlen_forward.register_fake
def _(q, k, v, cu_seqlens_q, cu_seqlens_k, max_sq, max_sk, causal, scale):
    _check_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_sq, max_sk)
    return torch.empty_like(q, memory_format=torch.contiguous_format), q.new_empty((q.shape[1], q.shape[0]),
                                                                                   dtype=torch.float32)


def _varlen_setup_context(ctx, inputs, output):
    q, k, v, cu_q, cu_k, max_sq, max_sk, causal, scale = inputs
    o, lse = output
    ctx.save_for_backward(q, k, v, o, lse, cu_q, cu_k)
    ctx.max_sq, ctx.max_sk, ctx.causal = max_sq, max_sk, causal
    ctx.scale = 1 / math.sqrt(HEAD_DIM) if scale <= 0 else scale
    ctx.set_materialize_grads(False)


def _varlen_backward(ctx, grad_o, grad_lse):
    q, k, v, o, lse, cu_q, cu_k = ctx.saved_tensors
    if grad_lse is not None:
        raise NotImplementedError("fav4::varlen_forward: the gradient through the LSE output is not implemented")
    if grad_o is None:
        return (None,) * 9
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    with torch.cuda.device(q.device):
        _runner().backward_varlen(q.contiguous(), k.contiguous(), v.contiguous(), o, grad_o.contiguous(), lse, dq,
                                  dk, dv, cu_q.contiguous(), cu_k.contiguous(), ctx.max_sq, ctx.max_sk, ctx.causal,
                                  ctx.scale)
    return dq, dk, dv, None, None, None, None, None, None


varlen_forward.register_autograd(_varlen_backward, setup_context=_varlen_setup_context)


def varlen_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, max_sq: int, max_sk: int, causal: bool = False,
                     scale: float | None = None, return_lse: bool = False):
    """O, or (O, LSE) when ``return_lse``, of packed sequences; differentiable in q, k, v."""
    o, lse = torch.ops.fav4.varlen_forward(q, k, v, cu_seqlens_q, cu_seqlens_k, max_sq, max_sk, causal,
                                           -1.0 if scale is None else scale)
    return (o, lse) if return_lse else o


def attention(q, k, v, causal: bool = False, config: int = 0, scale: float | None = None,
              return_lse: bool = False):
    """O, or (O, LSE) when ``return_lse``; differentiable in q, k, v (the LSE
    is always computed so that the backward pass can use it)."""
    o, lse = torch.ops.fav4.bshd_forward(q, k, v, causal, config, -1.0 if scale is None else scale, True)
    return (o, lse) if return_lse else o

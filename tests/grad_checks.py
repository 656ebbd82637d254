"""Comparison helpers shared by the GPU gradient tests."""
import torch


def dq_close(got, want):
    """dQ of the fused backward against another run of the same gradients: FP32
    reductions summed in a different order move a BF16 value by at most one ulp
    (rtol 2^-7), and where partial sums cancel by up to 1e-4 of the gradient's
    largest magnitude (atol)."""
    g, w = got.float(), want.float()
    return torch.allclose(g, w, rtol=2 ** -7, atol=1e-4 * w.abs().max().item() + 1e-6)

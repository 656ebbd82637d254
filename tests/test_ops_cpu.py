"""CPU tests of the PyTorch operator ``torch.ops.fav4.bshd_forward``: the
schema, and the fake (meta) implementation's shapes and argument checks under
FakeTensor tracing -- no GPU needed, no kernel runs."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from fav4_bshd import ops  # noqa: F401  (registers the operator)


def test_schema():
    schema = str(torch.ops.fav4.bshd_forward.default._schema)
    assert schema.startswith("fav4::bshd_forward(Tensor q, Tensor k, Tensor v, bool causal, SymInt config, "
                             "float scale, bool return_lse) -> (Tensor, Tensor)")


@pytest.mark.parametrize("return_lse", [True, False])
def test_fake_shapes(return_lse):
    with FakeTensorMode():
        q = torch.empty(3, 1000, 5, 128, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(3, 1537, 5, 128, dtype=torch.bfloat16, device="cuda")
        o, lse = torch.ops.fav4.bshd_forward(q, k, k, True, 0, -1.0, return_lse)
        assert o.shape == q.shape and o.dtype == torch.bfloat16 and o.device == q.device
        assert lse.dtype == torch.float32
        assert lse.shape == ((3, 5, 1000) if return_lse else (0,))


@pytest.mark.parametrize("case", ["dtype", "head_dim", "kv_mismatch", "heads", "config"])
def test_fake_rejects_invalid(case):
    with FakeTensorMode():
        q = torch.empty(2, 64, 4, 128, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(2, 64, 4, 128, dtype=torch.bfloat16, device="cuda")
        v = k
        config = 0
        if case == "dtype":
            q = q.to(torch.float16)
        elif case == "head_dim":
            q = torch.empty(2, 64, 4, 64, dtype=torch.bfloat16, device="cuda")
        elif case == "kv_mismatch":
            v = torch.empty(2, 65, 4, 128, dtype=torch.bfloat16, device="cuda")
        elif case == "heads":  # K/V heads must divide the query heads
            k = v = torch.empty(2, 64, 3, 128, dtype=torch.bfloat16, device="cuda")
        else:
            config = 4
        with pytest.raises(RuntimeError):
            torch.ops.fav4.bshd_forward(q, k, v, False, config, -1.0, False)


def test_varlen_schema_and_fake_shapes():
    schema = str(torch.ops.fav4.varlen_forward.default._schema)
    assert schema.startswith("fav4::varlen_forward(Tensor q, Tensor k, Tensor v, Tensor cu_seqlens_q, "
                             "Tensor cu_seqlens_k, SymInt max_sq, SymInt max_sk, bool causal, float scale)")
    with FakeTensorMode():
        q = torch.empty(900, 8, 128, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(700, 2, 128, dtype=torch.bfloat16, device="cuda")
        cu = torch.empty(4, dtype=torch.int32, device="cuda")
        o, lse = torch.ops.fav4.varlen_forward(q, k, k, cu, cu, 400, 300, True, -1.0)
        assert o.shape == q.shape and lse.shape == (8, 900) and lse.dtype == torch.float32
        with pytest.raises(RuntimeError):  # max_sq beyond total_q
            torch.ops.fav4.varlen_forward(q, k, k, cu, cu, 901, 300, True, -1.0)
        with pytest.raises(RuntimeError):  # heads not divisible
            torch.ops.fav4.varlen_forward(q, torch.empty(700, 3, 128, dtype=torch.bfloat16, device="cuda"),
                                          torch.empty(700, 3, 128, dtype=torch.bfloat16, device="cuda"), cu, cu, 400,
                                          300, True, -1.0)

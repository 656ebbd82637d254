"""GPU unit tests of the sm_100a building blocks, each exact.

* TMA BSHD tile load: the analogue of the reference's TDM probe
  (tests/bshd_tdm.hip:19-45) -- row stride heads*128, head offset (last head),
  zero fill of rows past the end -- for the 4-D map + 128-byte swizzle the
  attention kernel uses.
* UMMA S = A B^T (both K-major) and O = P V (P from TMEM, V MN-major): the two
  descriptor forms of the kernel, on small-integer inputs so every product and
  sum is exact in FP32.
* Bounded mbarrier wait: a wait on a barrier nobody arrives on gives up after
  its limit, sets the status word and lets the kernel finish.
"""
import ctypes as C

import pytest
import torch

import fav4_bshd as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def probe(cuda):
    return F.load_probe_library()


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("heads", [3, 8, 513])
@pytest.mark.parametrize("rows", [1, 17, 47, 64, 128, 200])
def test_tma_bshd_tile_load(probe, heads, rows):
    head = heads - 1
    r = torch.arange(rows, device="cuda").view(rows, 1, 1)
    h = torch.arange(heads, device="cuda").view(1, heads, 1)
    d = torch.arange(128, device="cuda").view(1, 1, 128)
    # integers < 256 are exact in BF16 (the reference used FP16 and % 1021)
    x = ((r * 137 + h * 71 + d * 13) % 251).to(torch.bfloat16).contiguous()
    out = torch.full((128, 128), -1.0, device="cuda", dtype=torch.bfloat16)
    assert probe.fav4_probe_tma_load(x.data_ptr(), out.data_ptr(), rows, heads, head, _stream()) == 0
    torch.cuda.synchronize()
    want = torch.zeros(128, 128, device="cuda", dtype=torch.bfloat16)
    n = min(rows, 128)
    want[:n] = x[:n, head]
    assert torch.equal(out, want)


def _small_ints(shape, gen):
    return torch.randint(-3, 4, shape, generator=gen, device="cuda").to(torch.bfloat16)


@pytest.mark.parametrize("seed", [0, 1])
def test_umma_qk_descriptor(probe, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    a = _small_ints((128, 128), gen)
    b = _small_ints((128, 128), gen)
    d = torch.full((128, 128), float("nan"), device="cuda")
    assert probe.fav4_probe_gemm_qk(a.data_ptr(), b.data_ptr(), d.data_ptr(), _stream()) == 0
    torch.cuda.synchronize()
    want = a.double() @ b.double().T
    assert torch.equal(d.double(), want)


@pytest.mark.parametrize("seed", [0, 1])
def test_umma_pv_descriptor_tmem_operand(probe, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    p = _small_ints((128, 128), gen)
    v = _small_ints((128, 128), gen)
    d = torch.full((128, 128), float("nan"), device="cuda")
    assert probe.fav4_probe_gemm_pv(p.data_ptr(), v.data_ptr(), d.data_ptr(), _stream()) == 0
    torch.cuda.synchronize()
    want = p.double() @ v.double()
    assert torch.equal(d.double(), want)


def test_bounded_wait_gives_up_and_reports(probe):
    assert probe.fav4_probe_status(1) >= 0  # clear
    out = torch.full((3,), -1, device="cuda", dtype=torch.int32)
    assert probe.fav4_probe_bounded_wait(20000, out.data_ptr(), _stream()) == 0  # 20 ms limit
    torch.cuda.synchronize()
    ok, waited_us, abort = out.tolist()
    assert ok == 0 and abort == 1
    assert 20000 <= waited_us < 2_000_000
    assert probe.fav4_probe_status(1) & 16
    assert probe.fav4_probe_status(0) == 0
    # the context is still usable
    x = torch.ones(4, device="cuda")
    assert float(x.sum()) == 4.0

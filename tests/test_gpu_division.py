"""The norm-fused projections divide by the RMS denominator with a correctly rounded reciprocal
and one fma correction (Markstein's theorem) instead of the general division sequence. The
reference divides in fp32 (gemma_dual.py:78, ``op.divide(xf, op.sqrt(var + eps))``), so the
replacement must agree with IEEE division bit for bit on the operand ranges the norm sees."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _div_check(a, b):
    from mlc_vla import _lib
    lib = _lib.load()
    out = torch.empty_like(a)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.pi0_div_check(ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                           ctypes.c_void_p(out.data_ptr()), a.numel(), ctypes.c_void_p(st))
    assert rc == 0
    torch.cuda.synchronize()
    return out


def test_division_matches_ieee():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    n = 1 << 24
    # numerators: fp16-representable magnitudes over the whole half range and random fp32;
    # denominators: sqrt(mean + eps) for eps = 1e-6 up to large activations
    a_half = (torch.randn(n, generator=g, device=dev) *
              torch.exp2(torch.randint(-24, 16, (n,), generator=g, device=dev).float())
              ).half().float()
    a_f32 = torch.randn(n, generator=g, device=dev) * 100.0
    b = torch.sqrt(torch.exp2(torch.rand(n, generator=g, device=dev) * 50.0 - 20.0) + 1e-6)
    for a in (a_half, a_f32):
        got = _div_check(a, b)
        want = a / b
        # includes ±0 and ±inf numerators (fp16 underflow / overflow): signed results must match
        bad = (got.view(torch.int32) != want.view(torch.int32)).sum().item()
        assert bad == 0, f"{bad} of {n} quotients differ from IEEE division"


def test_division_edge_values():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    dev = torch.device("cuda", 0)
    inf, nan = float("inf"), float("nan")
    a = torch.tensor([0.0, -0.0, 1.0, -1.0, 65504.0, -65504.0, 6.1035156e-05, 5.9604645e-08,
                      3.0, 1.0 / 3.0, inf, -inf, nan], device=dev)
    b = torch.tensor([1e-3, 1e-3, 1.0, 3.0, 1e-3, 7.0, 1.0000001, 0.999999, 1.7320508, 1e3, 0.5,
                      3.0, 2.0], device=dev)
    got, want = _div_check(a, b), a / b
    fin = torch.isfinite(want)
    assert torch.equal(got[fin].view(torch.int32), want[fin].view(torch.int32))
    assert torch.equal(torch.isnan(got), torch.isnan(want))
    assert torch.equal(got[torch.isinf(want)], want[torch.isinf(want)])

"""Failure path without a GPU fault: every wait inside the library's kernels is bounded. A wait
on a barrier phase that nothing completes gives up after about a second, records a timeout code
in a device error flag and lets the kernel return; the context stays usable for the next call."""
import ctypes
import time

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ERR_TIMEOUT = 3


def _wait(lib, err, arrive):
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.pi0_wait_check(ctypes.c_void_p(err.data_ptr()), arrive, st) == 0
    torch.cuda.synchronize()
    return int(err.item())


def test_bounded_wait_completes_or_reports_timeout():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from mlc_vla import _lib

    lib = _lib.load()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _wait(lib, err, 1) == 0          # the phase completes: no error
    t0 = time.perf_counter()
    assert _wait(lib, err, 0) == ERR_TIMEOUT  # nothing arrives: the wait gives up
    assert 0.5 < time.perf_counter() - t0 < 30
    # the context is still usable: an ordinary kernel runs and is correct
    a = torch.arange(1, 1025, dtype=torch.float32, device="cuda")
    b = torch.full_like(a, 4.0)
    out = torch.empty_like(a)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.pi0_div_check(ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                             ctypes.c_void_p(out.data_ptr()), a.numel(), st) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, a / b)

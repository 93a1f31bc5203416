"""pi0_linear_noalloc: the warp-level split-K projection with its scratch in static device
memory. Called through the C ABI and compared with the context-owning engine (pi0_linear,
engine 2) on the same inputs, two calls in a row each, so the second call runs on tickets the
first one left behind. For M < 256 the two use the same tiling and must agree bit for bit; for
M >= 256 engine 2 switches to 128 × 128 tiles without a split, so there they agree within
rounding. After a warm-up call, a call must not change the device's free memory. Collected
last so it also runs after every other GPU test."""
import ctypes

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

SHAPES = [(50, 1024, 2560), (50, 4096, 1024), (7, 2048, 96), (128, 1024, 512), (1, 256, 64),
          (300, 1024, 256)]


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_noalloc_matches_context_engine(dtype):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from gpu_common import config
    from mlc_vla import _lib
    from mlc_vla.runtime import Pi0Runtime
    from tests.golden import recipes

    lib = _lib.load()
    tdt = getattr(torch, dtype)
    code = _lib.DTYPE_CODE[dtype]
    rt = Pi0Runtime(config(recipes.MINI, dtype=dtype), device=0)
    dev = torch.device("cuda", 0)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator(device=dev).manual_seed(11)
    for M, K, N in SHAPES:
        x = torch.randn((M, K), generator=g, device=dev).to(tdt)
        w = (torch.randn((N, K), generator=g, device=dev) * 0.05).to(tdt)
        want = rt.linear(x, w, engine=2)
        ref = x.float() @ w.float().t()
        for _ in range(2):
            got = torch.full((M, N), float("nan"), dtype=tdt, device=dev)
            rc = lib.pi0_linear_noalloc(code, _ptr(x), M, K, _ptr(w), N, _ptr(got), st)
            assert rc == 0, rc
            torch.cuda.synchronize()
            assert torch.isfinite(got.float()).all()
            if M < 256:  # same engine, tiling and split rule as the context-owning call
                assert torch.equal(got, want), (M, K, N)
            else:
                tol = 1e-2 * ref.abs().max().item()
                assert (got.float() - want.float()).abs().max().item() <= tol, (M, K, N)
            err = (got.float() - ref).abs().max().item()
            assert err <= 1e-2 * ref.abs().max().item() + 2e-3, (M, K, N, err)
    # steady state: once warmed up, a call leaves the device's free memory unchanged
    M, K, N = SHAPES[0]
    x = torch.randn((M, K), generator=g, device=dev).to(tdt)
    w = torch.randn((N, K), generator=g, device=dev).to(tdt)
    got = torch.empty((M, N), dtype=tdt, device=dev)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(dev)[0]
    assert lib.pi0_linear_noalloc(code, _ptr(x), M, K, _ptr(w), N, _ptr(got), st) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(dev)[0] == free0
    assert rt.device_error() == 0
    rt.close()


def test_noalloc_rejects_oversize_and_bad_args():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from mlc_vla import _lib

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    x = torch.zeros((4, 64), dtype=torch.float16, device=dev)
    w = torch.zeros((2, 64), dtype=torch.float16, device=dev)
    y = torch.zeros((4, 2), dtype=torch.float16, device=dev)
    assert lib.pi0_linear_noalloc(_lib.PI0_F16, _ptr(x), 4, 63, _ptr(w), 2, _ptr(y), st) == _lib.PI0_ERR_INVALID
    assert lib.pi0_linear_noalloc(_lib.PI0_F32, _ptr(x), 4, 64, _ptr(w), 2, _ptr(y), st) == _lib.PI0_ERR_INVALID
    # offset pointers: x or w off a 16-byte boundary, y off a 4-byte boundary (refused on the
    # host, so no kernel runs)
    def off(t, nbytes):
        return ctypes.c_void_p(t.data_ptr() + nbytes)

    for args in ((off(x, 2), _ptr(w), _ptr(y)), (_ptr(x), off(w, 8), _ptr(y)),
                 (_ptr(x), _ptr(w), off(y, 2))):
        assert lib.pi0_linear_noalloc(_lib.PI0_F16, args[0], 4, 64, args[1], 2, args[2], st) == _lib.PI0_ERR_INVALID
    # a split-K shape whose partials exceed the static scratch (M·N·splits > 2^20 floats)
    M, K, N = 128, 8192, 4096
    xb = torch.zeros((M, K), dtype=torch.float16, device=dev)
    wb = torch.zeros((N, K), dtype=torch.float16, device=dev)
    yb = torch.zeros((M, N), dtype=torch.float16, device=dev)
    assert lib.pi0_linear_noalloc(_lib.PI0_F16, _ptr(xb), M, K, _ptr(wb), N, _ptr(yb), st) == _lib.PI0_ERR_UNSUPPORTED

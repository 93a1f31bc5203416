"""GPU: the GEMM engines (tcgen05/TMA and warp-level mma) against a plain PyTorch fp32 reference
of the same op, y = round(x·wᵀ), on shapes that exercise partial tiles in M, N and K."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt():
    from gpu_common import config
    from mlc_vla.runtime import Pi0Runtime
    from tests.golden import recipes

    return Pi0Runtime(config(recipes.MINI), device=0)


@pytest.mark.parametrize("engine", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (968, 2560, 2048), (200, 160, 320),
                                   (50, 1024, 4096), (777, 390, 96), (1000, 32768, 128),
                                   (50, 2560, 1024), (50, 8192, 1024), (50, 1024, 2048),
                                   (100, 160, 200), (8, 384, 128), (1, 3072, 1024),
                                   (968, 2048, 16384), (300, 1000, 4160)])
def test_linear_matches_torch_fp32(rt, engine, m, n, k):
    if engine == 2 and k % 32:
        pytest.skip("warp-level engine needs K % 32 == 0")
    if engine == 3 and (m > 128 or k > 16 * 4 * 64):
        pytest.skip("weight-streaming engine: M <= 128, K <= 4096")
    if engine == 1 and m < 128:
        pytest.skip("tile engine: M >= 128")
    if engine == 4 and (m < 128 or k <= 64):
        pytest.skip("split-K pair engine: M >= 128, K > 64")
    if engine == 5 and m < 128:
        pytest.skip("CTA-pair tile engine: M >= 128")
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    x = torch.randn((m, k), generator=g, device="cuda").half()
    w = (0.05 * torch.randn((n, k), generator=g, device="cuda")).half()
    y = rt.linear(x, w, engine=engine)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    ref = (x.float() @ w.float().T)
    err = (y.float() - ref).abs()
    tol = 1e-2 * ref.abs().max().item() + 2e-3
    assert err.max().item() <= tol, (err.max().item(), tol)
    rel = (err.norm() / ref.norm()).item()
    assert rel < 2e-3


@pytest.mark.parametrize("m,n,k", [(968, 32768, 2048), (200, 512, 192), (1000, 1280, 4160)])
def test_cta_pair_tiles_equal_single_cta_tiles(rt, m, n, k):
    """A 256-row tile on a CTA pair (cta_group::2) accumulates every output over K in the same
    order as a 128-row tile on one CTA: the two engines give the same bits."""
    g = torch.Generator(device="cuda").manual_seed(m + 3 * n + k)
    x = torch.randn((m, k), generator=g, device="cuda").half()
    w = (0.05 * torch.randn((n, k), generator=g, device="cuda")).half()
    y1 = rt.linear(x, w, engine=1)
    y5 = rt.linear(x, w, engine=5)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    assert torch.equal(y1, y5), (y1.float() - y5.float()).abs().max().item()


def test_engine_number_out_of_range_is_refused(rt):
    from mlc_vla import _lib

    x = torch.zeros((128, 64), dtype=torch.float16, device="cuda")
    w = torch.zeros((64, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(_lib.Pi0Error):
        rt.linear(x, w, engine=6)


def test_cta_pair_tiles_bf16():
    """The CTA-pair engine in a bfloat16 context (the MMA's operand type bits): equal to the
    single-CTA tiles bit for bit and within rounding of a torch fp32 product, at the prefill
    gate/up shape the automatic choice sends to it."""
    from gpu_common import config
    from mlc_vla.runtime import Pi0Runtime
    from tests.golden import recipes

    rt = Pi0Runtime(config(recipes.MINI, "bfloat16"), device=0)
    m, n, k = 968, 32768, 2048
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn((m, k), generator=g, device="cuda").bfloat16()
    w = (0.05 * torch.randn((n, k), generator=g, device="cuda")).bfloat16()
    y1 = rt.linear(x, w, engine=1)
    y5 = rt.linear(x, w, engine=5)
    y0 = rt.linear(x, w, engine=0)
    torch.cuda.synchronize()
    assert rt.device_error() == 0
    assert torch.equal(y1, y5) and torch.equal(y0, y5)
    ref = x.float() @ w.float().T
    rel = ((y5.float() - ref).norm() / ref.norm()).item()
    assert rel < 4e-3, rel
    rt.close()

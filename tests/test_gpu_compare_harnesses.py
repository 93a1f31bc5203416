"""GPU: the comparison harnesses of the reference (``compare_kv.py``, ``compare_loop.py``,
``compare_pad.py``, ``compare_quant.py``) run against this package and pass their gates (M1 ≡ M0
cosine ≥ 0.99; in-graph loop ≡ host loop ≥ 0.9999; padding masked ≥ 0.9999; quantised vs fp
≥ 0.97)."""

import pytest

pytestmark = pytest.mark.gpu


def test_compare_kv_dummy():
    from mlc_vla import compare_kv
    from mlc_vla.model.pi0 import Pi0Config

    cfg = Pi0Config(paligemma_variant="dummy", action_expert_variant="dummy", max_token_len=16,
                    action_horizon=4, dtype="float16")
    assert compare_kv.run(cfg, "cuda", loop_steps=3)


def test_compare_loop():
    from mlc_vla import compare_loop

    assert compare_loop.run("cuda", "float16", steps=4, seed=0)
    assert compare_loop.run("cuda", "bfloat16", steps=3, seed=1)


def test_compare_pad():
    from mlc_vla import compare_pad

    assert compare_pad.run("cuda", pad=5, seed=0)


@pytest.mark.parametrize("quant", ["q4f16_1", "q4bf16_1"])
def test_compare_quant(quant):
    """The reference quotes its 0.97 gate for int4 groups; q3f16_1 on these 64-wide dummy experts
    gives cosine 0.95 (seven levels per group), so only the q4 presets are gated here (q3's
    dequantisation is checked bit for bit in test_gpu_quant_model.py)."""
    from mlc_vla import compare_quant
    from mlc_vla.model.pi0 import Pi0Config

    cfg = Pi0Config(paligemma_variant="dummy", action_expert_variant="dummy", max_token_len=16,
                    action_horizon=4)
    assert compare_quant.run(cfg, "cuda", quant, seed=0)


@pytest.mark.parametrize("quant", [None, "q4f16_1"])
def test_bench_kv_dummy(quant):
    from mlc_vla import bench_kv
    from mlc_vla.model.pi0 import Pi0Config

    cfg = Pi0Config(paligemma_variant="dummy", action_expert_variant="dummy", max_token_len=16,
                    action_horizon=4)
    out = bench_kv.run(cfg, "cuda", steps=3, iters=3, quant=quant)
    assert out["prefill_ms"] > 0 and out["step_kv_ms"] > 0
    if quant is None:
        assert out["step_m0_ms"] > 0

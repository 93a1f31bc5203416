"""CPU: pin the oracle and the drop-in's host helpers to the reference's own outputs.

The fixtures in tests/golden/golden.npz were produced by tests/golden/make_golden.py from the
reference project's Python (its torch golden ``_SelfContainedRef`` and its ``sample.py``
helpers). Nothing here needs a GPU.
"""

import numpy as np
import pytest

from conftest import cosine, max_abs
from oracle import pi0_oracle as O
from tests.golden import recipes


def _cfg(kw, dtype):
    from mlc_vla.model.pi0 import Pi0Config

    return Pi0Config(**{**kw, "dtype": dtype})


@pytest.mark.parametrize("tag,kw", [("mini", recipes.MINI), ("dummy", recipes.DUMMY)])
def test_oracle_m1_matches_reference_torch_golden(golden, tag, kw):
    """prefill + denoise_step_kv (oracle, fp32) == the reference's _SelfContainedRef (M0)."""
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = _cfg(kw, "float32")
    params = O.random_params(backbone_named_params(cfg), seed=0)
    total = sum(float(np.sum(v, dtype=np.float64)) for v in params.values())
    assert total == pytest.approx(float(golden[f"{tag}_weights_sum"]), rel=0, abs=1e-9)
    inp = recipes.inputs(cfg, seed=1)
    for k, v in inp.items():
        assert float(np.sum(v, dtype=np.float64)) == pytest.approx(float(golden[f"{tag}_in_{k}_sum"]))
    p = O.prepare_params(params, "float32")
    pm = O.prefix_mask(cfg.prefix_len)
    keys, values = O.prefill(p, cfg, inp["prefix"], pm)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    v = O.denoise_step_kv(p, cfg, keys, values, inp["x_t"], inp["time_emb"], sc, ss, pm)
    ref = golden[f"{tag}_v_ref"]
    assert v.shape == ref.shape
    assert cosine(v, ref) >= 0.99999
    assert max_abs(v, ref) < 1e-5


def test_oracle_m0_matches_reference_torch_golden(golden):
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = _cfg(recipes.MINI, "float32")
    p = O.prepare_params(O.random_params(backbone_named_params(cfg), seed=0), "float32")
    inp = recipes.inputs(cfg, seed=1)
    v = O.denoise_step(p, cfg, inp["prefix"], inp["x_t"], inp["time_emb"])
    assert max_abs(v, golden["mini_v_ref"]) < 1e-5


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_oracle_m1_equals_m0_in_model_dtype(dtype):
    """compare_kv gate (python/mlc_vla/compare_kv.py:85-110) on the dtype-faithful oracle."""
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = _cfg(recipes.MINI, dtype)
    p = O.prepare_params(O.random_params(backbone_named_params(cfg), seed=0), dtype)
    inp = recipes.inputs(cfg, seed=1)
    pm = O.prefix_mask(cfg.prefix_len)
    keys, values = O.prefill(p, cfg, inp["prefix"], pm)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    v1 = O.denoise_step_kv(p, cfg, keys, values, inp["x_t"], inp["time_emb"], sc, ss, pm)
    v0 = O.denoise_step(p, cfg, inp["prefix"], inp["x_t"], inp["time_emb"])
    assert cosine(v0, v1) >= 0.999


def test_oracle_fp16_fixture_is_current(golden):
    """The committed fp16 oracle outputs (used by the GPU tests) match a fresh oracle run."""
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = _cfg(recipes.MINI, "float16")
    p = O.prepare_params(O.random_params(backbone_named_params(cfg), seed=0), "float16")
    inp = recipes.inputs(cfg, seed=1)
    pm = O.prefix_mask(cfg.prefix_len)
    keys, values = O.prefill(p, cfg, inp["prefix"], pm)
    assert np.array_equal(keys, golden["mini16_keys"])
    assert np.array_equal(values, golden["mini16_values"])


def test_host_helpers_bit_identical_to_reference(golden):
    from mlc_vla import sample
    from mlc_vla.openpi_ref import build_joint_additive_mask, sinusoidal_time_emb

    for off in (0, 7, 868, 968):
        c, s = sample.make_rope_np(50, 256, 10_000.0, offset=off)
        assert np.array_equal(c, golden[f"rope_s50_hd256_off{off}_cos"])
        assert np.array_equal(s, golden[f"rope_s50_hd256_off{off}_sin"])
    c, s = sample.make_rope_np(8, 64, 10_000.0, offset=64)
    assert np.array_equal(c, golden["rope_s8_hd64_off64_cos"])
    assert np.array_equal(sample.make_prefix_mask_np(968), golden["mask_p968_all"])
    assert np.array_equal(sample.make_prefix_mask_np(968, num_valid=868), golden["mask_p968_nv868"])
    assert np.array_equal(sample.make_prefix_mask_np(968, pad_mask=golden["mask_p968_pad_in"]),
                          golden["mask_p968_pad"])
    assert np.array_equal(np.concatenate(sample.make_time_embs(10, 1024), 0),
                          golden["time_embs_n10_w1024"])
    assert np.array_equal(np.concatenate(sample.make_time_embs(3, 128), 0),
                          golden["time_embs_n3_w128"])
    assert np.array_equal(sinusoidal_time_emb(0.7, 1024), golden["sinusoidal_t0.7_w1024"])
    assert np.array_equal(build_joint_additive_mask(6, 3), golden["joint_mask_p6_s3"])
    out = sample.euler_loop(lambda x, i: np.sin(x + i).astype(np.float32), golden["euler_x0"], 5)
    assert np.array_equal(out, golden["euler_out"])
    # the oracle's own copies of the tables agree too
    assert np.array_equal(O.time_embs(10, 1024), golden["time_embs_n10_w1024"])
    c, s = O.suffix_rope(type("C", (), {"suffix_len": 50, "rope_theta": 1e4,
                                         "vlm": type("V", (), {"head_dim": 256})})(), 868)
    assert np.array_equal(c, golden["rope_s50_hd256_off868_cos"])


def test_oracle_loop_equals_host_loop():
    """compare_loop gate (python/mlc_vla/compare_loop.py:56-60) on the oracle: fp32 identical."""
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = _cfg(recipes.MINI, "float32")
    p = O.prepare_params(O.random_params(backbone_named_params(cfg), seed=0), "float32")
    inp = recipes.inputs(cfg, seed=1)
    pm = O.prefix_mask(cfg.prefix_len)
    keys, values = O.prefill(p, cfg, inp["prefix"], pm)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    n = cfg.num_denoise_steps
    a = O.denoise_loop_kv(p, cfg, keys, values, inp["noise"], O.time_embs(n, cfg.action_expert.width),
                          sc, ss, pm)
    b = O.host_loop(p, cfg, keys, values, inp["noise"], sc, ss, pm, n)
    assert np.array_equal(a, b)


def test_oracle_pad_invariance():
    """compare_pad gate (python/mlc_vla/compare_pad.py:62-91): padded garbage prefix tokens
    masked out give the same v as the truncated prefix."""
    import dataclasses

    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    pad = 5
    full = _cfg({**recipes.MINI}, "float32")
    trunc = dataclasses.replace(full, max_token_len=full.max_token_len - pad)
    p = O.prepare_params(O.random_params(backbone_named_params(full), seed=0), "float32")
    rng = np.random.default_rng(0)
    P, V = full.prefix_len, trunc.prefix_len
    prefix = (0.02 * rng.standard_normal((1, P, full.vlm.width))).astype(np.float32)
    prefix[:, V:] = 10.0 * rng.standard_normal((1, pad, full.vlm.width))
    x_t = np.zeros((1, full.action_horizon, full.action_dim), np.float32)
    te = O.sinusoidal_time_emb(0.7, full.action_expert.width)

    def run(cfg, pre):
        pm = O.prefix_mask(cfg.prefix_len, num_valid=V)
        k, v = O.prefill(p, cfg, pre, pm)
        sc, ss = O.suffix_rope(cfg, V)
        return O.denoise_step_kv(p, cfg, k, v, x_t, te, sc, ss, pm)

    a = run(full, prefix)
    b = run(trunc, prefix[:, :V].copy())
    assert cosine(a, b) >= 0.9999


def test_embed_language_oracle_formula():
    """embed_language = table[id] · sqrt(width), the constant in the model dtype
    (pi0_model.py:101-104): sqrt(2048) is 45.25 in fp16 and bf16."""
    from oracle import pi0_oracle as O

    table = np.arange(4 * 2048, dtype=np.float32).reshape(4, 2048) / 4096.0
    out = O.embed_language(table, np.array([[2, 0]]), "float16")
    c = np.float32(np.float16(np.sqrt(2048.0)))
    assert c == np.float32(45.25)
    want = (np.float16(table[[2, 0]]).astype(np.float32) * c).astype(np.float16)
    assert np.array_equal(out.reshape(2, 2048), want)
    out32 = O.embed_language(table, np.array([1]), "float32")
    assert np.allclose(out32, table[1] * np.float32(np.sqrt(2048.0)))

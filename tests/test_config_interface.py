"""CPU: Pi0Config contract (port of the reference's python/tests/test_config_interface.py)."""

import json

import pytest


def test_default_config_derived_shapes():
    from mlc_vla.model.pi0 import Pi0Config

    cfg = Pi0Config()
    assert cfg.num_images == 3
    assert cfg.prefix_len == 3 * cfg.siglip.num_patches + cfg.max_token_len == 3 * 256 + 200
    assert cfg.suffix_len == cfg.action_horizon == 10
    assert cfg.attn_logits_dtype == "float32"
    assert cfg.vlm.head_dim == cfg.action_expert.head_dim


def test_from_openpi_config_reads_json_and_applies_overrides(tmp_path):
    from mlc_vla.model.pi0 import Pi0Config

    (tmp_path / "config.json").write_text(json.dumps({
        "action_dim": 7, "action_horizon": 5, "paligemma_variant": "dummy",
        "action_expert_variant": "dummy", "precision": "bfloat16"}))
    cfg = Pi0Config.from_openpi_config(str(tmp_path), dtype="float16", attn_logits_dtype="float16")
    assert (cfg.action_dim, cfg.action_horizon, cfg.paligemma_variant) == (7, 5, "dummy")
    assert cfg.dtype == "float16" and cfg.attn_logits_dtype == "float16"
    assert cfg.suffix_len == 5


def test_from_openpi_config_accepts_directory_or_file(tmp_path):
    from mlc_vla.model.pi0 import Pi0Config

    (tmp_path / "config.json").write_text(json.dumps(
        {"action_dim": 3, "action_horizon": 2, "paligemma_variant": "dummy",
         "action_expert_variant": "dummy"}))
    a = Pi0Config.from_openpi_config(str(tmp_path))
    b = Pi0Config.from_openpi_config(str(tmp_path / "config.json"))
    assert a.action_dim == b.action_dim == 3


def test_dual_expert_mismatch_rejected():
    from mlc_vla.model.pi0 import Pi0Config

    with pytest.raises(AssertionError):
        Pi0Config(paligemma_variant="gemma_2b", action_expert_variant="dummy")


def test_import_needs_no_tvm():
    import sys

    import mlc_vla.model.pi0  # noqa: F401
    import mlc_vla.sample  # noqa: F401

    assert "tvm" not in sys.modules

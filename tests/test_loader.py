"""The openpi checkpoint loader (``mlc_vla.model.pi0.pi0_loader``; reference
``python/mlc_vla/model/pi0/pi0_loader.py:83-203``).

* Its name map equals the reference loader's, entry for entry (target name, source keys in
  order, transform), for the small and the full π0.5 configuration: ``tests/golden/
  loader_map.json`` is the reference's own ``build_name_map`` output (``make_golden.py``).
* A checkpoint written in openpi names (safetensors, fp32 and bf16) loads back into the exact
  parameter table, and the loader reports missing keys and wrong shapes.
"""

import json
import os

import numpy as np
import pytest

from oracle import pi0_oracle as O
from tests.golden import recipes

HERE = os.path.dirname(os.path.abspath(__file__))


def _config(kw, dtype="float32"):
    from mlc_vla.model.pi0 import Pi0Config

    return Pi0Config(**{**kw, "dtype": dtype})


@pytest.mark.parametrize("label,kw", [("mini", recipes.MINI), ("full", recipes.FULL)])
def test_name_map_matches_reference(label, kw):
    from mlc_vla.model.pi0 import pi0_loader as L

    with open(os.path.join(HERE, "golden", "loader_map.json")) as f:
        ref = json.load(f)[label]
    ours = L.build_name_map(_config(kw))
    assert sorted(ours) == sorted(ref)
    kinds = {"_concat_gate_up": L.concat_gate_up, "_conv_to_linear": L.conv_to_linear,
             "<lambda>": None}
    for name, spec in ours.items():
        assert spec.keys == ref[name]["keys"], name
        assert spec.fn is kinds[ref[name]["fn"]], name


def test_table_is_covered_by_the_map():
    from mlc_vla.model.pi0 import pi0_loader as L
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = _config(recipes.FULL)
    names = set(L.build_name_map(cfg))
    assert all(n in names for n, _ in backbone_named_params(cfg))


def _write(tmp_path, sd, dtype):
    import torch
    from safetensors.torch import save_file

    path = os.path.join(tmp_path, "model.safetensors")
    save_file({k: torch.from_numpy(np.ascontiguousarray(v)).to(dtype) for k, v in sd.items()},
              path)
    return path


def test_round_trip_through_safetensors(tmp_path):
    import torch

    from mlc_vla.model.pi0 import pi0_loader as L
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = _config(recipes.MINI)
    table = backbone_named_params(cfg)
    params = O.random_params(table, seed=0)
    sd = L.to_openpi(cfg, params)
    assert "paligemma_with_expert.gemma_expert.model.layers.1.mlp.up_proj.weight" in sd
    assert ("paligemma_with_expert.gemma_expert.model.layers.0.input_layernorm.dense.bias"
            in sd)
    src = L.load_safetensors(_write(str(tmp_path), sd, torch.float32))
    got = L.load_params(cfg, src, named_params=table)
    assert set(got) == {n for n, _ in table}
    for n, _ in table:
        assert got[n].dtype == np.float32 and np.array_equal(got[n], params[n]), n
    arrays = L.param_list(table, got)
    assert len(arrays) == len(table)

    # gate rows first, then up rows (reference pi0_loader.py:56-58)
    gu = got["backbone.layers.0.mlp.1.gate_up_proj.weight"]
    pre = "paligemma_with_expert.gemma_expert.model.layers.0.mlp."
    f = gu.shape[0] // 2
    assert np.array_equal(gu[:f], sd[pre + "gate_proj.weight"])
    assert np.array_equal(gu[f:], sd[pre + "up_proj.weight"])


def test_bf16_checkpoint_widens_then_casts(tmp_path):
    import torch

    from mlc_vla.model.pi0 import pi0_loader as L
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = _config(recipes.MINI, "float16")
    table = backbone_named_params(cfg)
    params = O.random_params(table, seed=3)
    sd = L.to_openpi(cfg, params)
    src = L.load_safetensors(_write(str(tmp_path), sd, torch.bfloat16))
    got = L.load_params(cfg, src, named_params=table)
    for n, _ in table:
        want = torch.from_numpy(np.ascontiguousarray(params[n])).to(torch.bfloat16).float()
        want = want.numpy().astype(np.float16)
        assert got[n].dtype == np.float16 and np.array_equal(got[n], want), n


def test_missing_key_and_wrong_shape_are_reported():
    from mlc_vla.model.pi0 import pi0_loader as L
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = _config(recipes.MINI)
    table = backbone_named_params(cfg)
    sd = L.to_openpi(cfg, O.random_params(table, seed=0))
    gone = dict(sd)
    del gone["paligemma_with_expert.paligemma.model.language_model.layers.1.self_attn.k_proj.weight"]
    with pytest.raises(KeyError):
        L.load_params(cfg, gone, named_params=table)
    bad = dict(sd)
    bad["action_in_proj.weight"] = np.zeros((3, 3), np.float32)
    with pytest.raises(ValueError):
        L.load_params(cfg, bad, named_params=table)


def test_conv_to_linear_order():
    from mlc_vla.model.pi0 import pi0_loader as L

    conv = np.arange(2 * 3 * 4 * 4, dtype=np.float32).reshape(2, 3, 4, 4)
    lin = L.conv_to_linear(conv)
    assert lin.shape == (2, 48)
    # element (h, c, i, j) of the conv lands at column (i·p + j)·c_count + c
    for h, c, i, j in [(0, 0, 0, 0), (1, 2, 3, 1), (0, 1, 2, 3)]:
        assert lin[h, (i * 4 + j) * 3 + c] == conv[h, c, i, j]

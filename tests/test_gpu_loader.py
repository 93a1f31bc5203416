"""GPU: a model loaded from an openpi-named checkpoint (``pi0_loader``; reference
``python/mlc_vla/model/pi0/pi0_loader.py:159-203``) runs the path and matches the committed
oracle outputs of the same seeded weights (the checkpoint is written from those weights in
openpi names, fp32, so loading is exact)."""

import os

import numpy as np
import pytest

from conftest import cosine, max_abs
from gpu_common import config
from oracle import pi0_oracle as O
from tests.golden import recipes

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def test_checkpoint_loaded_model_matches_golden(tmp_path, golden):
    from safetensors.torch import save_file

    from mlc_vla.model.pi0 import pi0_loader as L
    from mlc_vla.model.pi0.pi0_model import backbone_named_params
    from mlc_vla.runtime import Pi0Runtime

    cfg = config(recipes.MINI)
    table = backbone_named_params(cfg)
    sd = L.to_openpi(cfg, O.random_params(table, seed=0))
    path = os.path.join(str(tmp_path), "model.safetensors")
    save_file({k: torch.from_numpy(np.ascontiguousarray(v, np.float32)) for k, v in sd.items()},
              path)
    params = L.load_params(cfg, L.load_safetensors(path), named_params=table)
    rt = Pi0Runtime(cfg, device=0)
    assert [n for n, _ in rt.named_params] == [n for n, _ in table]
    rt.bind(rt.to_params(L.param_list(table, params)))
    inp = recipes.inputs(cfg, seed=1)
    pm = O.prefix_mask(cfg.prefix_len)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    k, v = rt.prefill(inp["prefix"], pm)
    vt = rt.denoise_step_kv(k, v, inp["x_t"], inp["time_emb"], sc, ss, pm).float().cpu().numpy()
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    x = rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm).float().cpu().numpy()
    assert rt.device_error() == 0
    for out, ref, what in ((vt, golden["mini16_v"], "step"), (x, golden["mini16_loop"], "loop")):
        c, m = cosine(out, ref), max_abs(out, ref)
        print(f"[parity] checkpoint-loaded {what}: cos={c:.7f} max_abs={m:.3e}")
        assert c >= 0.9995 and m <= 2e-2, (what, c, m)
    rt.close()

"""GPU: the model with group-quantised Linear weights (q4f16_1, q4bf16_1, q3f16_1; SURVEY C4,
``quant.py:117-266``, ``compile_quant.quantize_params`` ``compile_quant.py:71-103``).

Every Linear weight is quantised with the reference quantiser's semantics (the oracle's restated
``GroupQuantize``), the packed (q_weight, q_scale, bias) table is bound through the C ABI, and
prefill + denoise_loop_kv are compared with the oracle run on the dequantised weights. The library
dequantises bit-exactly (``test_gpu_quantiser_bit_exact``), so the comparison carries the same
tolerances as the unquantised model.
"""

import numpy as np
import pytest

from conftest import cosine, max_abs
from gpu_common import config
from oracle import pi0_oracle as O
from oracle import quant_oracle as Q
from tests.golden import recipes

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _quantised_params(cfg, preset, seed=0):
    """(list in the quantised table's order, oracle parameters with dequantised weights)."""
    from mlc_vla.model.pi0.pi0_model import backbone_named_params
    from mlc_vla.quant import PRESETS

    raw = O.random_params(backbone_named_params(cfg), seed=seed)
    model_dtype = PRESETS[preset].model_dtype
    table = backbone_named_params(cfg, quant=PRESETS[preset])
    arrays, deq = [], dict(raw)
    for name, spec in table:
        if name.endswith(".q_weight"):
            base = name[: -len(".q_weight")]
            w = O.rnd(raw[base + ".weight"], model_dtype)
            qw, qs = Q.quantize(w, preset)
            arrays.append(qw)
            deq[base + ".weight"] = Q.dequantize(qw, qs, preset, w.shape[1])
            deq.setdefault("_scales", {})[base] = qs
        elif name.endswith(".q_scale"):
            base = name[: -len(".q_scale")]
            arrays.append(deq["_scales"][base])
        else:
            arrays.append(raw[name])
    deq.pop("_scales", None)
    return table, arrays, deq


@pytest.mark.parametrize("preset", ["q4f16_1", "q3f16_1", "q4bf16_1"])
def test_quantised_model_matches_oracle_on_dequantised_weights(preset):
    from mlc_vla.quant import PRESETS
    from mlc_vla.runtime import Pi0Runtime

    q = PRESETS[preset]
    cfg = config(recipes.MINI, q.model_dtype)
    table, arrays, deq = _quantised_params(cfg, preset)
    rt = Pi0Runtime(cfg, device=0, quant=q)
    assert [n for n, _ in rt.named_params] == [n for n, _ in table]
    rt.bind(rt.to_params(arrays))

    inp = recipes.inputs(cfg, seed=1)
    pm = O.prefix_mask(cfg.prefix_len)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    k, v = rt.prefill(inp["prefix"], pm)
    x = rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm).float().cpu().numpy()
    assert rt.device_error() == 0

    p = O.prepare_params(deq, q.model_dtype)
    ko, vo = O.prefill(p, cfg, inp["prefix"], pm)
    xo = O.denoise_loop_kv(p, cfg, ko, vo, inp["noise"], te, sc, ss, pm)
    c, m = cosine(x, xo), max_abs(x, xo)
    print(f"[parity] quantised {preset}: cos={c:.7f} max_abs={m:.3e}")
    cos_min, tol = (0.9995, 2e-2) if q.model_dtype == "float16" else (0.999, 8e-2)
    assert c >= cos_min and m <= tol, (preset, c, m)
    rt.close()

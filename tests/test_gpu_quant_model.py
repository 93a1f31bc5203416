"""GPU: the model with group-quantised Linear weights (q4f16_1, q4bf16_1, q3f16_1; the
quantised serving configuration, ``quant.py:117-266``, ``compile_quant.quantize_params`` ``compile_quant.py:71-103``).

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


def _quantised_params(cfg, preset, seed=0, scale=1.0):
    """(list in the quantised table's order, oracle parameters with dequantised weights). `scale`
    multiplies every Linear weight before quantisation."""
    from mlc_vla.model.pi0.pi0_model import backbone_named_params
    from mlc_vla.quant import PRESETS

    raw = O.random_params(backbone_named_params(cfg), seed=seed)
    model_dtype = PRESETS[preset].model_dtype
    table = backbone_named_params(cfg, quant=PRESETS[preset])
    arrays, deq = [], dict(raw)
    for name, spec in table:
        if name.endswith(".q_weight"):
            base = name[: -len(".q_weight")]
            w = O.rnd(raw[base + ".weight"] * scale, model_dtype)
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


def _suffix_inputs(cfg, batch, seed=3):
    rng = np.random.default_rng(seed)
    nvs = [int(v) for v in rng.integers(cfg.prefix_len // 2, cfg.prefix_len + 1, size=batch)]
    pm = np.concatenate([O.prefix_mask(cfg.prefix_len, nv) for nv in nvs], 0)
    rope = [O.suffix_rope(cfg, nv) for nv in nvs]
    sc = np.concatenate([r[0] for r in rope], 0)
    ss = np.concatenate([r[1] for r in rope], 0)
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    return pm, sc, ss, te


def _fused_vs_bind_time(cfg, q, qarrays, deq_arrays, batch):
    """Runs the quantised runtime (q blocks dequantised inside the weight-streaming GEMMs) and an
    unquantised runtime bound to the dequantised weights on the same inputs; returns both
    outputs of prefill, denoise_step_kv and denoise_loop_kv."""
    from mlc_vla.runtime import Pi0Runtime

    import os

    rq = Pi0Runtime(cfg, device=0, quant=q, max_batch=batch)
    rq.bind(rq.to_params(qarrays))
    # the same kernels as the quantised context (the per-kernel chain), so the two agree bit for bit
    os.environ.pop("PI0_STEP_KERNEL", None)
    rf = Pi0Runtime(cfg, device=0, max_batch=batch)
    rf.bind(rf.to_params(deq_arrays))
    inp = recipes.inputs(cfg, seed=1, batch=batch)
    pm, sc, ss, te = _suffix_inputs(cfg, batch)
    out = []
    for rt in (rq, rf):
        k, v = rt.prefill(inp["prefix"], pm)
        vt = rt.denoise_step_kv(k, v, inp["x_t"], inp["time_emb"], sc, ss, pm)
        x = rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm)
        torch.cuda.synchronize()
        assert rt.device_error() == 0
        out.append([t.clone() if isinstance(t, torch.Tensor) else t.torch.clone()
                    for t in (k, v, vt, x)])
    rq.close()
    rf.close()
    return out


@pytest.mark.parametrize("preset,scale", [("q4f16_1", 1.0), ("q3f16_1", 1.0), ("q4bf16_1", 1.0),
                                          ("q4f16_1", 1e-3), ("q3f16_1", 1e-3)])
def test_fused_group_dequant_is_bit_exact(preset, scale):
    """The denoise path's weight-streaming GEMMs read the group-quantised blocks and dequantise
    them in shared memory (w = (code − max_int)·scale, ``quant.py:176-193``); the result must be
    bit-identical to the same model run on weights dequantised ahead of time. scale 1e-3 puts the
    group scales and the dequantised fp16 weights in the subnormal range."""
    from mlc_vla.quant import PRESETS

    q = PRESETS[preset]
    cfg = config(recipes.MINI, q.model_dtype)
    table, arrays, deq = _quantised_params(cfg, preset, scale=scale)
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    deq_arrays = [deq[n] for n, _ in backbone_named_params(cfg)]
    (kq, vq, vtq, xq), (kf, vf, vtf, xf) = _fused_vs_bind_time(cfg, q, arrays, deq_arrays, 1)
    assert torch.equal(kq, kf) and torch.equal(vq, vf)
    assert torch.equal(vtq, vtf), (vtq - vtf).abs().max().item()
    assert torch.equal(xq, xf), (xq - xf).abs().max().item()


@pytest.mark.parametrize("preset,batch", [("q4f16_1", 1), ("q4f16_1", 2), ("q3f16_1", 2)])
def test_fused_group_dequant_full_width(preset, batch):
    """Every pi0.5 width (2 layers): projections with K = 1024, 2048 and 4096, split-K clusters,
    and 64- (batch 1) and 128-row (batch 2, M = 100) activation tiles. The weights are quantised
    on the GPU (``pi0_quantize_weight``, bit-exact with the reference quantiser)."""
    from mlc_vla.model.pi0.pi0_model import backbone_named_params
    from mlc_vla.quant import PRESETS
    from mlc_vla.runtime import dequantize_weight, quantize_weight

    q = PRESETS[preset]
    cfg = config(recipes.FULL2, q.model_dtype)
    gen = torch.Generator(device="cuda").manual_seed(11)
    raw = {n: (torch.randn(tuple(s.shape), generator=gen, device="cuda") * 0.02).half()
           for n, s in backbone_named_params(cfg)}
    qarrays, deq = [], dict(raw)
    for name, spec in backbone_named_params(cfg, quant=q):
        if name.endswith(".q_weight"):
            base = name[: -len(".q_weight")]
            w = raw[base + ".weight"]
            qw, qs = quantize_weight(w, q)
            qarrays += [qw, qs]
            deq[base + ".weight"] = dequantize_weight(qw, qs, q, w.shape[1])
        elif not name.endswith(".q_scale"):
            qarrays.append(raw[name])
    deq_arrays = [deq[n] for n, _ in backbone_named_params(cfg)]
    (kq, vq, vtq, xq), (kf, vf, vtf, xf) = _fused_vs_bind_time(cfg, q, qarrays, deq_arrays, batch)
    assert torch.equal(kq, kf) and torch.equal(vq, vf)
    assert torch.equal(vtq, vtf), (vtq - vtf).abs().max().item()
    assert torch.equal(xq, xf), (xq - xf).abs().max().item()

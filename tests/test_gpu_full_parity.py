"""GPU parity at the benchmarked size: the full 18-layer π0.5 fp16 model against the oracle.

The model the bench times (both experts at every π0.5 width, 18 layers, P=968, S=50, D=32,
10 Euler steps) is compared with oracle outputs committed by ``tests/golden/make_full_fixtures.py``
(the oracle needs tens of seconds per request at this size). Weights are regenerated here from
the same seeded draws (``recipes.seeded_weights``), inputs from ``recipes.inputs``.

* C2, batch 1, all prefix positions valid: ``prefill`` K/V at 17 sampled positions of every
  layer and the per-layer L2 norms of the whole caches, one ``denoise_step_kv`` and the 10-step
  ``denoise_loop_kv`` (reference ``pi0_model.py:128-194``).
* C3, batch 8, the last 100 prefix positions padded (mask from ``prefix_pad``, suffix RoPE offset
  868; ``sample.py:50-64,139-187``): the 10-step loop of every request.

Each runs with the reference's attention-logits setting (``attn_logits_dtype``): ``float32``, its
default, and ``float16``, its tensor-core option; the oracle computes the same setting.
Tolerances: actions cosine ≥ 0.9995 and max-abs ≤ 2e-2; K/V cosine ≥ 0.99999 and max-abs ≤ 1 %
of the largest magnitude; cache norms within 1e-3 relative.
"""

import os

import numpy as np
import pytest
import torch

from conftest import cosine, max_abs
from oracle import pi0_oracle as O
from tests.golden import recipes
from tests.golden.make_full_fixtures import C3_BATCH, C3_VALID, PATH

pytestmark = pytest.mark.gpu

COS, MAXABS = 0.9995, 2e-2


def _np(t):
    return t.float().cpu().numpy()


def _check(out, ref, cos=COS, mx=MAXABS, what=""):
    c, m = cosine(out, ref), max_abs(out, ref)
    print(f"[full parity] {what}: cos={c:.7f} max_abs={m:.3e}")
    assert c >= cos and m <= mx, (what, c, m)


@pytest.fixture(scope="module")
def fixtures():
    if not os.path.exists(PATH):
        pytest.skip("tests/golden/full_pi05.npz not generated")
    return dict(np.load(PATH))


@pytest.fixture(scope="module")
def weights():
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = Pi0Config(**{**recipes.FULL, "dtype": "float16"})
    named = backbone_named_params(cfg)
    raw = recipes.seeded_weights(named, seed=0)
    dev = torch.device("cuda", 0)
    out = [torch.from_numpy(raw.pop(n)).to(dev).to(torch.float16) for n, _ in named]
    return out


@pytest.fixture(scope="module", params=["float32", "float16"])
def model(request, weights):
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.runtime import Pi0Runtime

    cfg = Pi0Config(**{**recipes.FULL, "dtype": "float16", "attn_logits_dtype": request.param})
    rt = Pi0Runtime(cfg, device=0, max_batch=C3_BATCH)
    rt.bind(weights)
    yield cfg, rt, "f32" if request.param == "float32" else "f16"
    rt.close()


def test_c2_prefill_step_loop(model, fixtures):
    cfg, rt, tag = model
    if f"c2_{tag}_v" not in fixtures:
        pytest.skip(f"no {tag} fixtures")
    P = cfg.prefix_len
    inp = recipes.inputs(cfg, seed=1, batch=1)
    pm = O.prefix_mask(P)
    sc, ss = O.suffix_rope(cfg, P)
    k, v = rt.prefill(inp["prefix"], pm)
    pos = torch.from_numpy(fixtures["positions"]).to(k.device)
    ks = _np(k[:, 0, 0].index_select(1, pos))
    vs = _np(v[:, 0, 0].index_select(1, pos))
    kr, vr = fixtures[f"c2_{tag}_keys_s"], fixtures[f"c2_{tag}_values_s"].astype(np.float32)
    _check(ks, kr, 0.99999, 1e-2 * np.abs(kr).max(), f"{tag} keys (sampled positions)")
    _check(vs, vr, 0.99999, 1e-2 * np.abs(vr).max(), f"{tag} values (sampled positions)")
    kl2 = torch.linalg.vector_norm(k.double().flatten(1), dim=1).cpu().numpy()
    vl2 = torch.linalg.vector_norm(v.double().flatten(1), dim=1).cpu().numpy()
    np.testing.assert_allclose(kl2, fixtures[f"c2_{tag}_keys_l2"], rtol=1e-3)
    np.testing.assert_allclose(vl2, fixtures[f"c2_{tag}_values_l2"], rtol=1e-3)
    v1 = _np(rt.denoise_step_kv(k, v, inp["x_t"], inp["time_emb"], sc, ss, pm))
    _check(v1, fixtures[f"c2_{tag}_v"], what=f"{tag} denoise_step_kv")
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    x = _np(rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm))
    _check(x, fixtures[f"c2_{tag}_loop"], what=f"{tag} denoise_loop_kv")
    assert rt.device_error() == 0


def test_c3_batch8_padded_loop(model, fixtures):
    cfg, rt, tag = model
    if f"c3_{tag}_loop" not in fixtures:
        pytest.skip(f"no {tag} fixtures")
    P = cfg.prefix_len
    inp = recipes.inputs(cfg, seed=2, batch=C3_BATCH)
    pm = np.concatenate([O.prefix_mask(P, C3_VALID)] * C3_BATCH, 0)
    sc, ss = O.suffix_rope(cfg, C3_VALID)
    sc, ss = np.concatenate([sc] * C3_BATCH, 0), np.concatenate([ss] * C3_BATCH, 0)
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    k, v = rt.prefill(inp["prefix"], pm)
    x = _np(rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm))
    ref = fixtures[f"c3_{tag}_loop"]
    for b in range(C3_BATCH):
        _check(x[b:b + 1], ref[b:b + 1], what=f"{tag} batch-8 padded request {b}")
    assert rt.device_error() == 0

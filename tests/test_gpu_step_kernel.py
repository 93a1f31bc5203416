"""The persistent denoise step (one launch per step, denoise_step.cuh; opt-in with
PI0_STEP_KERNEL=1) against the oracle and against the per-kernel chain, the default path.

Runs at every π0.5 width with two layers (FULL2), batch 1, both attention-logits settings:
``denoise_step_kv`` and the 10-step ``denoise_loop_kv`` (reference pi0_model.py:142-194) within
the fp16 tolerance (cosine ≥ 0.9995, max-abs ≤ 2e-2) of the oracle and of the chain, the host-
stepped loop bit-identical to the in-graph loop, and a step that launches a handful of kernels
(time MLP and modulations, the key conversion, the step) instead of about a hundred.
"""

import os

import numpy as np
import pytest
import torch

from conftest import cosine, max_abs
from gpu_common import Model, config
from oracle import pi0_oracle as O
from tests.golden import recipes

pytestmark = pytest.mark.gpu

COS, MAXABS = 0.9995, 2e-2


def _np(t):
    return t.float().cpu().numpy()


def _check(out, ref, what):
    c, m = cosine(out, ref), max_abs(out, ref)
    print(f"[step kernel] {what}: cos={c:.7f} max_abs={m:.3e}")
    assert c >= COS and m <= MAXABS, (what, c, m)


def _launches(rt):
    return rt.lib.pi0_launch_count(rt._ctx)


@pytest.mark.parametrize("logits", ["float32", "float16"])
def test_step_kernel_matches_oracle_and_chain(logits):
    cfg = config(recipes.FULL2, attn_logits_dtype=logits)
    os.environ["PI0_STEP_KERNEL"] = "1"
    try:
        m = Model(cfg)
    finally:
        del os.environ["PI0_STEP_KERNEL"]
    inp = m.inputs(seed=3)
    nv = 900
    pm = O.prefix_mask(cfg.prefix_len, nv)
    sc, ss = O.suffix_rope(cfg, nv)
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    k, v = m.rt.prefill(inp["prefix"], pm)
    torch.cuda.synchronize()
    n0 = _launches(m.rt)
    vs = _np(m.rt.denoise_step_kv(k, v, inp["x_t"], inp["time_emb"], sc, ss, pm))
    n_step = _launches(m.rt) - n0
    assert m.rt.device_error() == 0
    assert n_step <= 8, f"{n_step} launches for one denoise step: the persistent step did not run"
    x = _np(m.rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm))
    assert m.rt.device_error() == 0
    ko, vo = m.oracle_kv(inp["prefix"], pm)
    _check(vs, O.denoise_step_kv(m.p, cfg, ko, vo, inp["x_t"], inp["time_emb"], sc, ss, pm),
           f"{logits} step vs oracle")
    _check(x, O.denoise_loop_kv(m.p, cfg, ko, vo, inp["noise"], te, sc, ss, pm),
           f"{logits} loop vs oracle")
    # host-stepped loop == in-graph loop, bit for bit (the same launches)
    xh = inp["noise"].astype(np.float32)
    for i in range(cfg.num_denoise_steps):
        vv = _np(m.rt.denoise_step_kv(k, v, xh.astype(np.float16), te[i:i + 1], sc, ss, pm))
        xh = xh + (-1.0 / cfg.num_denoise_steps) * vv
    assert np.array_equal(xh, x)
    # the per-kernel chain on the same weights and inputs
    from mlc_vla.runtime import Pi0Runtime

    rt2 = Pi0Runtime(cfg, device=0)
    rt2.bind(m.params)
    n0 = _launches(rt2)
    vs2 = _np(rt2.denoise_step_kv(k, v, inp["x_t"], inp["time_emb"], sc, ss, pm))
    assert _launches(rt2) - n0 > 10  # 5 per layer plus action in/out, time MLP, keys
    x2 = _np(rt2.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm))
    _check(vs, vs2, f"{logits} step: persistent vs chain")
    _check(x, x2, f"{logits} loop: persistent vs chain")
    rt2.close()

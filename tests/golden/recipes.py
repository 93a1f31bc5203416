"""Seeded test configurations and inputs shared by the fixture generator and the tests.

``MINI`` is the CPU-runnable small dual-expert model of the benchmark configuration list
(prefix width 256 / 2 layers / 4 q heads / 1 kv head / head_dim 64 / GeGLU 1024; action
width 128 / GeGLU 512; P=64, S=8, D=8, 3 Euler steps). ``DUMMY`` is the reference tests'
configuration (``python/tests/conftest.py:21-28``: dummy experts, max_token_len 8 → P=776,
horizon 4, 3 steps). ``FULL2`` has every π0.5 width (2048 / 1024, MLP 16384 / 4096, 8 heads,
head_dim 256, P=968, S=50, D=32) but only 2 layers, so the oracle finishes in seconds.
"""

import numpy as np

MINI = dict(paligemma_variant="mini_vlm", action_expert_variant="mini_action", image_keys=(),
            max_token_len=64, action_horizon=8, action_dim=8, num_denoise_steps=3)
DUMMY = dict(paligemma_variant="dummy", action_expert_variant="dummy", max_token_len=8,
             action_horizon=4, num_denoise_steps=3)
FULL2 = dict(paligemma_variant="gemma_2b_2l", action_expert_variant="gemma_300m_2l",
             action_horizon=50, action_dim=32, num_denoise_steps=10)
FULL = dict(action_horizon=50, action_dim=32, num_denoise_steps=10)


def inputs(cfg, seed=1, batch=1):
    """prefix_embs, x_t, time_emb (sinusoidal at t=0.7) and noise; N(0,1) draws from
    ``default_rng(seed)`` in that order."""
    from oracle.pi0_oracle import sinusoidal_time_emb

    rng = np.random.default_rng(seed)
    prefix = rng.standard_normal((batch, cfg.prefix_len, cfg.vlm.width)).astype(np.float32)
    x_t = rng.standard_normal((batch, cfg.action_horizon, cfg.action_dim)).astype(np.float32)
    noise = rng.standard_normal((batch, cfg.action_horizon, cfg.action_dim)).astype(np.float32)
    te = sinusoidal_time_emb(0.7, cfg.action_expert.width)
    return {"prefix": prefix, "x_t": x_t, "time_emb": te, "noise": noise}


def seeded_weights(named_params, seed=0, scale=0.02, threads=None):
    """N(0, scale²) fp32 weights in parameter-table order, fast enough for the 2.4 B-parameter
    π0.5 model: entry i is drawn from its own ``default_rng([seed, i])`` (float32 normals), so
    the values do not depend on the number of threads that draw them. Integer entries are
    zeros."""
    from concurrent.futures import ThreadPoolExecutor
    import os

    def draw(item):
        i, (_, spec) = item
        shape = tuple(int(s) for s in spec.shape)
        if str(spec.dtype).startswith(("int", "uint")):
            return np.zeros(shape, spec.dtype)
        w = np.random.default_rng([seed, i]).standard_normal(shape, dtype=np.float32)
        w *= np.float32(scale)
        return w

    with ThreadPoolExecutor(threads or os.cpu_count() or 1) as ex:
        vals = list(ex.map(draw, enumerate(named_params)))
    return {name: v for (name, _), v in zip(named_params, vals)}

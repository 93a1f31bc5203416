"""Prefix padding is masked out: the reference's ``python/mlc_vla/compare_pad.py``. Two models
with the same weights differ only in prefix length by `pad`; the longer one gets large random
garbage in its last `pad` prefix positions, masked with the pad mask (and the suffix RoPE offset
at the valid length). Its v_t must equal the shorter model's (cosine ≥ 0.9999).

    python -m mlc_vla.compare_pad --target cuda [--pad 5] [--seed 0]
"""

from __future__ import annotations

import argparse

import numpy as np

from mlc_vla._compare import cosine, in_order, m1_step, max_abs, random_weights
from mlc_vla.compile import compile_model
from mlc_vla.model.pi0 import Pi0Config
from mlc_vla.openpi_ref import sinusoidal_time_emb

_FUNCS = ["prefill", "denoise_step_kv"]


def _run(config, target, weights, prefix, num_valid):
    ex, npar = compile_model(config, target, functions=_FUNCS)
    params = ex.to_params(in_order(npar, weights))
    x_t = np.zeros((1, config.action_horizon, config.action_dim), np.float32)
    te = sinusoidal_time_emb(0.7, config.action_expert.width)
    return m1_step(ex, params, config, prefix, x_t, te, num_valid).astype(np.float32)


def run(target: str = "cuda", pad: int = 5, seed: int = 0, dtype: str = "float16") -> bool:
    base = dict(paligemma_variant="dummy", action_expert_variant="dummy", action_horizon=4,
                dtype=dtype)
    cfg_full = Pi0Config(**base, max_token_len=16)
    cfg_trunc = Pi0Config(**base, max_token_len=16 - pad)
    P, V = cfg_full.prefix_len, cfg_trunc.prefix_len
    assert P - V == pad
    W = cfg_full.vlm.width
    rng = np.random.default_rng(seed)
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    weights = random_weights(backbone_named_params(cfg_full), rng)  # same shapes for both
    prefix = (0.02 * rng.standard_normal((1, P, W))).astype(np.float32)
    prefix[:, V:, :] = 10.0 * rng.standard_normal((1, pad, W)).astype(np.float32)
    v_full = _run(cfg_full, target, weights, prefix, num_valid=V)
    v_trunc = _run(cfg_trunc, target, weights, prefix[:, :V, :].copy(), num_valid=V)
    cos = cosine(v_full, v_trunc)
    print(f"[compare_pad] P={P} V={V} pad={pad}  cosine={cos:.6f} "
          f"max_abs_diff={max_abs(v_full, v_trunc):.3e}")
    ok = cos >= 0.9999
    print(f"[compare_pad] {'PASS' if ok else 'FAIL'} (padded garbage tokens masked out)")
    return ok


def main():
    ap = argparse.ArgumentParser(description="prefix padding masked out")
    ap.add_argument("--target", default="cuda")
    ap.add_argument("--pad", type=int, default=5)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    raise SystemExit(0 if run(args.target, args.pad, args.seed) else 1)


if __name__ == "__main__":
    main()

"""M1 (prefill + denoise_step_kv) against M0 (the joint denoise_step), the reference's
``python/mlc_vla/compare_kv.py``: same random weights and inputs, the two paths must agree
(cosine ≥ 0.99; here they are bit-identical by construction), optionally over an N-step Euler loop.

    python -m mlc_vla.compare_kv --target cuda [--dtype float16|bfloat16] [--dummy] [--loop N]
"""

from __future__ import annotations

import argparse

import numpy as np

from mlc_vla._compare import cosine, in_order, m1_step, max_abs, on_device_dtype, random_weights
from mlc_vla.compile import compile_model
from mlc_vla.model.pi0 import Pi0Config
from mlc_vla.sample import euler_loop, make_time_embs

_FUNCS = ["denoise_step", "prefill", "denoise_step_kv"]


def run(config: Pi0Config, target: str = "cuda", loop_steps: int = 0, cublas=None,
        seed: int = 0) -> bool:
    config = on_device_dtype(config)
    ex, npar = compile_model(config, target, functions=_FUNCS, cublas=cublas)
    rng = np.random.default_rng(seed)
    params = ex.to_params(in_order(npar, random_weights(npar, rng)))
    prefix = rng.standard_normal((1, config.prefix_len, config.vlm.width)).astype(np.float32)
    x_t = rng.standard_normal((1, config.action_horizon, config.action_dim)).astype(np.float32)
    te = make_time_embs(1, config.action_expert.width)[0]
    v0 = ex["denoise_step"](prefix, x_t, te, params).numpy()
    v1 = m1_step(ex, params, config, prefix, x_t, te, config.prefix_len)
    cos = cosine(v0, v1)
    print(f"[compare_kv] M0 vs M1 step: shape={v0.shape} cosine={cos:.6f} "
          f"max_abs_diff={max_abs(v0, v1):.3e}")
    ok = cos >= 0.99
    if loop_steps > 0:
        tes = make_time_embs(loop_steps, config.action_expert.width)
        a0 = euler_loop(lambda x, i: ex["denoise_step"](prefix, x, tes[i], params).numpy(), x_t,
                        loop_steps)
        a1 = euler_loop(lambda x, i: m1_step(ex, params, config, prefix, x, tes[i],
                                             config.prefix_len), x_t, loop_steps)
        lcos = cosine(a0, a1)
        print(f"[compare_kv] {loop_steps}-step loop cosine={lcos:.6f} "
              f"max_abs_diff={max_abs(a0, a1):.3e}")
        ok = ok and lcos >= 0.99
    print(f"[compare_kv] {'PASS' if ok else 'FAIL'} (M1 == M0)")
    return ok


def main():
    ap = argparse.ArgumentParser(description="M1 K/V path against the M0 joint step")
    ap.add_argument("--target", default="cuda")
    ap.add_argument("--dtype", default=None, help="override config.dtype (float16 / bfloat16)")
    ap.add_argument("--dummy", action="store_true", help="small experts, quick check")
    ap.add_argument("--loop", type=int, default=0, help="also compare an N-step Euler loop")
    ap.add_argument("--cublas", action=argparse.BooleanOptionalAction, default=None)
    args = ap.parse_args()
    kw = dict(paligemma_variant="dummy", action_expert_variant="dummy") if args.dummy else {}
    config = Pi0Config(**kw)
    if args.dtype:
        config.dtype = args.dtype
    raise SystemExit(0 if run(config, args.target, args.loop, args.cublas) else 1)


if __name__ == "__main__":
    main()

"""In-graph Euler loop (``sample_graph``, one ``denoise_loop_kv``) against the host loop
(``sample``, one ``denoise_step_kv`` per step), the reference's ``python/mlc_vla/compare_loop.py``:
cosine ≥ 0.9999 in 16-bit dtypes (≥ 0.99999 in fp32 there); here the two are bit-identical.

    python -m mlc_vla.compare_loop --target cuda [--dtype float16] [--steps 4] [--seed 0]
"""

from __future__ import annotations

import argparse

import numpy as np

from mlc_vla._compare import cosine, in_order, max_abs, random_weights
from mlc_vla.model.pi0 import Pi0Config
from mlc_vla.sample import PiZeroRunner


def run(target: str = "cuda", dtype: str = "float16", steps: int = 4, seed: int = 0) -> bool:
    config = Pi0Config(paligemma_variant="dummy", action_expert_variant="dummy",
                       max_token_len=16, action_horizon=4, dtype=dtype, num_denoise_steps=steps)
    runner = PiZeroRunner(config, target)
    rng = np.random.default_rng(seed)
    params = runner.to_params(in_order(runner.named_params, random_weights(runner.named_params, rng)))
    prefix = (0.02 * rng.standard_normal((1, config.prefix_len, config.vlm.width))).astype(np.float32)
    noise = rng.standard_normal((1, config.action_horizon, config.action_dim)).astype(np.float32)
    x_host = runner.sample(params, prefix, noise=noise, num_steps=steps)
    x_graph = runner.sample_graph(params, prefix, noise=noise)
    cos = cosine(x_host, x_graph)
    print(f"[compare_loop] steps={steps} dtype={dtype}  cosine={cos:.6f} "
          f"max_abs_diff={max_abs(x_host, x_graph):.3e}")
    ok = cos >= (0.99999 if dtype == "float32" else 0.9999)
    print(f"[compare_loop] {'PASS' if ok else 'FAIL'} (in-graph loop == host loop)")
    return ok


def main():
    ap = argparse.ArgumentParser(description="in-graph Euler loop against the host loop")
    ap.add_argument("--target", default="cuda")
    ap.add_argument("--dtype", default="float16")
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    raise SystemExit(0 if run(args.target, args.dtype, args.steps, args.seed) else 1)


if __name__ == "__main__":
    main()

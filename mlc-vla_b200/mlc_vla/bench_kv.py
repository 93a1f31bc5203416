"""Latency of the exported functions, the reference's ``python/mlc_vla/bench_kv.py``: prefill,
one denoise_step_kv (M1), one denoise_step (M0), and the N-step totals, with random weights.
Times are device times from CUDA events (warm calls averaged over ``--iters``). With
``--quant`` the quantised M1 path is measured instead (no M0).

    python -m mlc_vla.bench_kv --target cuda [--dtype float16] [--steps 10] [--iters 30]
        [--dummy] [--quant q4f16_1]

The repository's ``bench.py`` is the benchmark of record (chunks/s, roofline, e2e); this tool
keeps the reference's per-function view.
"""

from __future__ import annotations

import argparse
import dataclasses

import numpy as np
import torch

from mlc_vla._compare import in_order, on_device_dtype, random_weights
from mlc_vla.compile import compile_model
from mlc_vla.model.pi0 import Pi0Config
from mlc_vla.sample import make_prefix_mask_np, make_rope_np, make_time_embs


def _time_ms(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def run(config: Pi0Config, target: str = "cuda", steps: int = 10, iters: int = 30, quant=None,
        seed: int = 0) -> dict:
    config = on_device_dtype(config)
    q = None
    if quant:
        from mlc_vla.quant import get_quant

        q = get_quant(quant)
        config = dataclasses.replace(config, dtype=q.model_dtype)
    funcs = ["prefill", "denoise_step_kv"] + ([] if q else ["denoise_step"])
    ex, npar = compile_model(config, target, functions=funcs, quant=q)
    rng = np.random.default_rng(seed)
    if q is None:
        params = ex.to_params(in_order(npar, random_weights(npar, rng)))
    else:
        from mlc_vla.model.pi0.pi0_model import backbone_named_params
        from mlc_vla.runtime import quantize_weight, to_device

        fp = random_weights(backbone_named_params(config), rng)
        arrays = []
        for name, _ in npar:
            if name.endswith(".q_weight"):
                w = to_device(fp[name[: -len(".q_weight")] + ".weight"], q.model_dtype, ex.device)
                arrays += quantize_weight(w, q)
            elif not name.endswith(".q_scale"):
                arrays.append(fp[name])
        params = ex.to_params(arrays)
    dev = ex.device
    dt = torch.float16 if config.dtype == "float16" else torch.bfloat16
    prefix = torch.randn((1, config.prefix_len, config.vlm.width), device=dev).to(dt)
    x_t = torch.randn((1, config.action_horizon, config.action_dim), device=dev).to(dt)
    te = torch.from_numpy(make_time_embs(1, config.action_expert.width)[0]).to(dev, dt)
    pm = torch.from_numpy(make_prefix_mask_np(config.prefix_len)).to(dev)
    c, s = make_rope_np(config.suffix_len, config.vlm.head_dim, config.rope_theta,
                        offset=config.prefix_len)
    sc, ss = torch.from_numpy(c).to(dev), torch.from_numpy(s).to(dev)
    ex.bind(params)
    kv = ex.prefill(prefix, pm)
    out = {"prefill_ms": _time_ms(lambda: ex.prefill(prefix, pm, keys=kv[0], values=kv[1]), iters),
           "step_kv_ms": _time_ms(lambda: ex.denoise_step_kv(kv[0], kv[1], x_t, te, sc, ss, pm),
                                  iters)}
    tag = "[bench-quant]" if q else "[bench]"
    print(f"{tag} prefill            : {out['prefill_ms']:8.3f} ms")
    print(f"{tag} denoise_step_kv(M1): {out['step_kv_ms']:8.3f} ms/step")
    total_m1 = out["prefill_ms"] + steps * out["step_kv_ms"]
    print(f"{tag} {steps}-step total  M1 (prefill+{steps}x): {total_m1:8.3f} ms")
    if q is None:
        out["step_m0_ms"] = _time_ms(lambda: ex.denoise_step(prefix, x_t, te), iters)
        print(f"{tag} denoise_step   (M0): {out['step_m0_ms']:8.3f} ms/step")
        print(f"{tag} {steps}-step total  M0 ({steps}x joint)   : {steps * out['step_m0_ms']:8.3f} ms")
        print(f"{tag} per-step speedup M0/M1 = {out['step_m0_ms'] / max(out['step_kv_ms'], 1e-6):.2f}x")
    return out


def main():
    ap = argparse.ArgumentParser(description="latency of prefill / denoise_step_kv / denoise_step")
    ap.add_argument("--target", default="cuda")
    ap.add_argument("--dtype", default=None)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--iters", type=int, default=30)
    ap.add_argument("--dummy", action="store_true")
    ap.add_argument("--quant", default=None, help="quantisation preset (e.g. q4f16_1)")
    args = ap.parse_args()
    kw = dict(paligemma_variant="dummy", action_expert_variant="dummy") if args.dummy else {}
    config = Pi0Config(**kw, action_horizon=50, action_dim=32)
    if args.dtype:
        config = dataclasses.replace(config, dtype=args.dtype)
    run(config, args.target, args.steps, args.iters, args.quant)


if __name__ == "__main__":
    main()

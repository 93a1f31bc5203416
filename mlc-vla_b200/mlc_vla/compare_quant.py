"""Group-quantised model against the floating-point model, the reference's
``python/mlc_vla/compare_quant.py``: the same fp source weights run (a) as they are and (b)
quantised with a preset; v_t of prefill + denoise_step_kv must keep cosine ≥ 0.97. With
``--ckpt`` the source weights come from an openpi safetensors checkpoint through ``pi0_loader``.

    python -m mlc_vla.compare_quant --target cuda [--quant q4bf16_1] [--dummy] [--ckpt PATH]
"""

from __future__ import annotations

import argparse

import numpy as np

from mlc_vla._compare import cosine, in_order, m1_step, max_abs, random_weights
from mlc_vla.compile import compile_model
from mlc_vla.model.pi0 import Pi0Config
from mlc_vla.model.pi0.pi0_model import backbone_named_params
from mlc_vla.openpi_ref import sinusoidal_time_emb
from mlc_vla.quant import get_quant
from mlc_vla.runtime import quantize_weight

_FUNCS = ["prefill", "denoise_step_kv"]


def run(config: Pi0Config, target: str = "cuda", quant_name: str = "q4bf16_1", seed: int = 0,
        ckpt=None) -> bool:
    import dataclasses

    quant = get_quant(quant_name)
    config = dataclasses.replace(config, dtype=quant.model_dtype)
    fp_table = backbone_named_params(config)
    if ckpt:
        from mlc_vla.model.pi0 import pi0_loader

        src = pi0_loader.load_params(config, pi0_loader.load_safetensors(ckpt), named_params=fp_table,
                                     dtype="float32")
    else:
        src = random_weights(fp_table, np.random.default_rng(seed))
    rng = np.random.default_rng(seed + 7)
    prefix = (0.02 * rng.standard_normal((1, config.prefix_len, config.vlm.width))).astype(np.float32)
    x_t = rng.standard_normal((1, config.action_horizon, config.action_dim)).astype(np.float32)
    te = sinusoidal_time_emb(0.7, config.action_expert.width).astype(np.float32)

    ex_fp, np_fp = compile_model(config, target, functions=_FUNCS)
    fp_params = ex_fp.to_params(in_order(np_fp, src))
    v_fp = m1_step(ex_fp, fp_params, config, prefix, x_t, te, config.prefix_len)
    fp_bytes = sum(t.numel() * t.element_size() for t in fp_params)
    del ex_fp

    ex_q, np_q = compile_model(config, target, functions=_FUNCS, quant=quant)
    by_name = dict(zip([n for n, _ in np_fp], fp_params))
    arrays = []
    for name, _ in np_q:
        if name.endswith(".q_weight"):
            arrays += quantize_weight(by_name[name[: -len(".q_weight")] + ".weight"], quant)
        elif not name.endswith(".q_scale"):
            arrays.append(by_name[name])
    q_params = ex_q.to_params(arrays)
    v_q = m1_step(ex_q, q_params, config, prefix, x_t, te, config.prefix_len)
    q_bytes = sum(t.numel() * t.element_size() for t in q_params)

    cos = cosine(v_fp, v_q)
    print(f"[compare_quant] quant={quant_name} shape={v_fp.shape} cosine={cos:.6f} "
          f"max_abs_diff={max_abs(v_fp, v_q):.3e}")
    print(f"[compare_quant] param bytes: fp={fp_bytes / 1e6:.1f}MB  quant={q_bytes / 1e6:.1f}MB  "
          f"ratio={fp_bytes / max(q_bytes, 1):.2f}x")
    ok = cos >= 0.97
    print(f"[compare_quant] {'PASS' if ok else 'FAIL'} (threshold=0.97)")
    return ok


def main():
    ap = argparse.ArgumentParser(description="group-quantised model against the fp model")
    ap.add_argument("--target", default="cuda")
    ap.add_argument("--quant", default="q4bf16_1")
    ap.add_argument("--dummy", action="store_true", help="small experts, quick check")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--ckpt", default=None, help="openpi safetensors checkpoint (optional)")
    args = ap.parse_args()
    kw = dict(paligemma_variant="dummy", action_expert_variant="dummy") if args.dummy else {}
    ok = run(Pi0Config(**kw), args.target, args.quant, args.seed, args.ckpt)
    raise SystemExit(0 if ok else 1)


if __name__ == "__main__":
    main()

"""Generate the full-size π0.5 fixtures (tests/golden/full_pi05.npz) with the CPU oracle.

    python tests/golden/make_full_fixtures.py [--modes float32,float16] [--threads N]

The benchmarked model — 18 layers of both experts at every π0.5 width (2048 / 1024, MLP
16384 / 4096, 8 q heads / 1 kv head × 256, P=968, S=50, D=32, 10 Euler steps), fp16 — takes the
oracle tens of seconds per request, too long to recompute inside every GPU test run, so its
outputs are computed once here and committed. Weights are ``recipes.seeded_weights`` (seed 0,
N(0, 0.02), regenerated bit-identically by the GPU test); inputs are ``recipes.inputs``.

For each attention-logits dtype in ``--modes`` (the reference's ``attn_logits_dtype``:
``float32``, its default, and ``float16``, its tensor-core option), the file holds:

* C2 (batch 1, all 968 prefix positions valid, suffix RoPE offset 968, seed 1 inputs):
  ``prefill`` keys and values at 17 sampled positions of every layer, the per-layer L2 norms of
  the whole key and value caches, one ``denoise_step_kv`` output at t = 0.7, and the 10-step
  ``denoise_loop_kv`` output;
* C3 (batch 8, the last 100 prefix positions padded, suffix RoPE offset 868, seed 2 inputs):
  the 10-step ``denoise_loop_kv`` output of every request.

Follows the reference functions ``pi0_model.py:128-194`` (prefill, denoise_step_kv,
denoise_loop_kv) and ``sample.py:50-64,139-187`` (pad mask, RoPE offset = #valid) through
``oracle/pi0_oracle.py``.
"""

from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
for _p in (REPO, os.path.join(REPO, "mlc-vla_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

PATH = os.path.join(HERE, "full_pi05.npz")
C3_BATCH, C3_VALID = 8, 868


def sample_positions(P):
    """17 prefix positions spread over the cache, first and last included."""
    return np.unique(np.concatenate([np.arange(0, P, 61), [P - 1]])).astype(np.int64)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--modes", default="float32,float16")
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    args = ap.parse_args()
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(args.threads)
    except ImportError:
        pass
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_model import backbone_named_params
    from oracle import pi0_oracle as O
    from tests.golden import recipes

    out = dict(np.load(PATH)) if os.path.exists(PATH) else {}
    base = Pi0Config(**{**recipes.FULL, "dtype": "float16"})
    t0 = time.time()
    raw = recipes.seeded_weights(backbone_named_params(base), seed=0)
    p = O.prepare_params(raw, "float16")
    del raw
    print(f"[full] weights {time.time() - t0:.1f}s", flush=True)
    P, S = base.prefix_len, base.action_horizon
    pos = sample_positions(P)
    out["positions"] = pos
    for mode in args.modes.split(","):
        cfg = Pi0Config(**{**recipes.FULL, "dtype": "float16", "attn_logits_dtype": mode})
        tag = "f32" if mode == "float32" else "f16"
        te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
        # ---- C2 ----
        inp = recipes.inputs(cfg, seed=1, batch=1)
        pm = O.prefix_mask(P)
        sc, ss = O.suffix_rope(cfg, P)
        t0 = time.time()
        keys, values = O.prefill(p, cfg, inp["prefix"], pm)
        t1 = time.time()
        out[f"c2_{tag}_keys_s"] = keys[:, 0, 0, pos]
        out[f"c2_{tag}_values_s"] = values[:, 0, 0, pos].astype(np.float16)
        out[f"c2_{tag}_keys_l2"] = np.sqrt(np.sum(keys.astype(np.float64) ** 2, axis=(1, 2, 3, 4)))
        out[f"c2_{tag}_values_l2"] = np.sqrt(np.sum(values.astype(np.float64) ** 2,
                                                    axis=(1, 2, 3, 4)))
        out[f"c2_{tag}_v"] = O.denoise_step_kv(p, cfg, keys, values, inp["x_t"], inp["time_emb"],
                                               sc, ss, pm)
        t2 = time.time()
        out[f"c2_{tag}_loop"] = O.denoise_loop_kv(p, cfg, keys, values, inp["noise"], te, sc, ss,
                                                  pm)
        t3 = time.time()
        print(f"[full] {mode} C2: prefill {t1 - t0:.1f}s, step {t2 - t1:.1f}s, "
              f"loop {t3 - t2:.1f}s", flush=True)
        # ---- C3 ----
        inp = recipes.inputs(cfg, seed=2, batch=C3_BATCH)
        pm = O.prefix_mask(P, C3_VALID)
        sc, ss = O.suffix_rope(cfg, C3_VALID)
        xs = []
        for b in range(C3_BATCH):
            k, v = O.prefill(p, cfg, inp["prefix"][b:b + 1], pm)
            xs.append(O.denoise_loop_kv(p, cfg, k, v, inp["noise"][b:b + 1], te, sc, ss, pm))
            print(f"[full] {mode} C3 request {b} done ({time.time() - t3:.1f}s)", flush=True)
        out[f"c3_{tag}_loop"] = np.concatenate(xs, 0)
        np.savez_compressed(PATH, **out)
        print(f"[full] wrote {PATH} ({os.path.getsize(PATH) / 1e3:.1f} kB)", flush=True)


if __name__ == "__main__":
    main()

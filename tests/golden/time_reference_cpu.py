"""Time the reference's own CPU model beside the numpy oracle, on this host (needs the reference
checkout; it cannot run on a GPU box, where the reference is absent).

    python tests/golden/time_reference_cpu.py [--reference <root of the reference checkout>]

The reference's CPU implementation of the path is ``openpi_ref._SelfContainedRef``
(``python/mlc_vla/openpi_ref.py:92-214``): a torch re-statement of openpi's joint (M0) denoise
step, prefix and suffix through both experts in one pass. The full π0.5 configuration (18
layers, P = 968, S = 50) is built with seeded N(0, 0.02) weights in fp32 and one ``denoise``
call is timed with every host thread; the oracle's ``denoise_step`` (the numpy port the bench's
CPU baseline runs) is timed on the same weights and inputs. Prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
for _p in (REPO, os.path.join(REPO, "mlc-vla_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    args = ap.parse_args()
    import torch

    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_model import backbone_named_params
    from oracle import pi0_oracle as O
    from tests.golden import make_golden as G
    from tests.golden import recipes

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref = G.load_reference(args.reference)
    cfg = Pi0Config(**{**recipes.FULL, "dtype": "float32"})
    params = recipes.seeded_weights(backbone_named_params(cfg), seed=0)
    sd = G.to_openpi_state_dict(ref, cfg, params)
    model = ref.openpi_ref._SelfContainedRef(cfg, sd, "cpu", torch.float32)
    inp = recipes.inputs(cfg, seed=1)
    t0 = time.perf_counter()
    v_ref = model.denoise(inp["prefix"], inp["x_t"], inp["time_emb"])
    t_ref = time.perf_counter() - t0
    del model, sd
    p32 = O.prepare_params(params, "float32")
    t0 = time.perf_counter()
    v_port = O.denoise_step(p32, cfg, inp["prefix"], inp["x_t"], inp["time_emb"])
    t_port = time.perf_counter() - t0
    print(json.dumps({
        "what": "one joint (M0) denoise step, pi0.5 full size, fp32, N(0,0.02) weights",
        "threads": threads,
        "reference_SelfContainedRef_s": round(t_ref, 2),
        "oracle_port_s": round(t_port, 2),
        "port_over_reference": round(t_port / t_ref, 3),
        "cosine_port_vs_reference": round(O.cosine(v_port, v_ref), 8),
        "max_abs_port_vs_reference": float(O.max_abs(v_port, v_ref)),
    }))


if __name__ == "__main__":
    main()

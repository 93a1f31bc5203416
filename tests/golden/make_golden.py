"""Generate the golden fixtures under tests/golden/ from the reference project.

Run here (where the read-only reference checkout exists), never on the GPU box:

    python tests/golden/make_golden.py --reference /path/to/mlc-vla

(or set MLC_VLA_REFERENCE to the reference checkout instead of passing --reference)

What it does:

1. Imports the reference's own Python (``python/mlc_vla/openpi_ref.py``, ``sample.py``,
   ``model/pi0/pi0_config.py``, ``model/pi0/pi0_loader.py``) behind stub package modules,
   because the reference's ``mlc_vla/model/pi0/__init__.py`` and ``compile.py`` import TVM,
   which is not installed. Nothing from TVM is executed.
2. Records the reference host helpers' outputs (RoPE tables, prefix masks, time embeddings,
   Euler loop) so the drop-in's restatements are checked bit for bit.
3. For the small dual-expert configuration (``mini``: prefix width 256 / 2 layers / 4 heads /
   head_dim 64, action width 128, P=64, S=8, D=8) and for the reference tests' ``dummy``
   configuration (P=776, S=4), builds N(0, 0.02) weights (seed 0) in the parameter-table
   order, converts them to openpi state-dict names with the reference's own loader map
   (``pi0_loader.build_name_map``), and runs the reference's torch golden
   ``_SelfContainedRef.denoise`` (M0 joint, fp32). Its output is the pin for the oracle's
   prefill + denoise_step_kv (M1) and denoise_step (M0), which must agree to cosine
   ≥ 0.99999 here before the fixture is written.
4. Writes the dtype-faithful fp16 oracle outputs of the ``mini`` configuration, which the
   GPU tests compare against.
5. Writes ``loader_map.json``: the reference loader's complete name map (``build_name_map``:
   target name -> source keys and the transform's name) for the ``mini`` and the full π0.5
   configuration, the pin of this package's checkpoint loader. ``--loader-map-only`` writes
   just this file.
"""

from __future__ import annotations

import argparse
import dataclasses
import importlib
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def load_reference(ref_root: str):
    """Import the reference's TVM-free modules under the name ``mlc_vla`` and hand them back.

    Our own package is also called ``mlc_vla``; its modules are moved out of ``sys.modules``
    while the reference loads and restored afterwards.
    """
    py = os.path.join(ref_root, "python", "mlc_vla")
    saved = {k: sys.modules.pop(k) for k in list(sys.modules)
             if k == "mlc_vla" or k.startswith("mlc_vla.")}
    try:
        def pkg(name, path):
            m = types.ModuleType(name)
            m.__path__ = [path]
            sys.modules[name] = m
            return m

        pkg("mlc_vla", py)
        pkg("mlc_vla.model", os.path.join(py, "model"))
        pi0 = pkg("mlc_vla.model.pi0", os.path.join(py, "model", "pi0"))
        cfgmod = importlib.import_module("mlc_vla.model.pi0.pi0_config")
        pi0.Pi0Config = cfgmod.Pi0Config
        pi0.GemmaExpertConfig = cfgmod.GemmaExpertConfig
        comp = types.ModuleType("mlc_vla.compile")
        comp._device_for = comp.compile_model = None
        sys.modules["mlc_vla.compile"] = comp
        ns = types.SimpleNamespace(
            config=cfgmod,
            openpi_ref=importlib.import_module("mlc_vla.openpi_ref"),
            sample=importlib.import_module("mlc_vla.sample"),
            loader=importlib.import_module("mlc_vla.model.pi0.pi0_loader"),
        )
    finally:
        for k in [k for k in sys.modules if k == "mlc_vla" or k.startswith("mlc_vla.")]:
            del sys.modules[k]
        sys.modules.update(saved)
    return ns


def to_openpi_state_dict(ref, config, params):
    """Map MLC-named parameters to openpi names with the reference's loader map, and check
    that the loader rebuilds every MLC parameter from the produced state dict."""
    import torch

    name_map = ref.loader.build_name_map(config)
    heads = ("action_in_proj", "action_out_proj", "time_mlp_in", "time_mlp_out")
    wanted = {k for k in name_map if k.startswith("backbone.") or k.split(".")[0] in heads}
    assert wanted == set(params), (sorted(wanted ^ set(params))[:5])
    sd = {}
    for name in wanted:
        spec = name_map[name]
        arr = params[name]
        if len(spec.keys) == 1:
            sd[spec.keys[0]] = arr
        else:  # gate_up = concat(gate, up) along rows
            f = arr.shape[0] // 2
            sd[spec.keys[0]], sd[spec.keys[1]] = arr[:f], arr[f:]
    for name in wanted:
        rebuilt = name_map[name].build(sd)
        assert np.array_equal(rebuilt, params[name]), name
    return {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)) for k, v in sd.items()}


def write_loader_map(ref):
    """The reference loader's name map for the mini and the full configuration, as JSON (the
    map reads only the depth, the vision depth and the π0.5 flag of the configuration it gets)."""
    import json

    from mlc_vla.model.pi0 import Pi0Config
    from tests.golden import recipes

    maps = {}
    for label, kw in (("mini", recipes.MINI), ("full", recipes.FULL)):
        config = Pi0Config(**kw)
        maps[label] = {name: {"keys": list(spec.keys), "fn": spec.fn.__name__}
                       for name, spec in ref.loader.build_name_map(config).items()}
    path = os.path.join(HERE, "loader_map.json")
    with open(path, "w") as f:
        json.dump(maps, f, indent=0, sort_keys=True)
    print("wrote", path, {k: len(v) for k, v in maps.items()})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MLC_VLA_REFERENCE"),
                    help="the reference checkout (default: $MLC_VLA_REFERENCE)")
    ap.add_argument("--loader-map-only", action="store_true")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set MLC_VLA_REFERENCE")

    ref = load_reference(args.reference)
    sys.path.insert(0, os.path.join(REPO, "mlc-vla_b200"))
    sys.path.insert(0, REPO)
    write_loader_map(ref)
    if args.loader_map_only:
        return
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_model import backbone_named_params
    from oracle import pi0_oracle as O
    from tests.golden import recipes

    out = {}
    # ---- host helpers, straight from the reference ----
    s = ref.sample
    for off in (0, 7, 868, 968):
        c, sn = s.make_rope_np(50, 256, 10_000.0, offset=off)
        out[f"rope_s50_hd256_off{off}_cos"], out[f"rope_s50_hd256_off{off}_sin"] = c, sn
    c, sn = s.make_rope_np(8, 64, 10_000.0, offset=64)
    out["rope_s8_hd64_off64_cos"], out["rope_s8_hd64_off64_sin"] = c, sn
    out["mask_p968_all"] = s.make_prefix_mask_np(968)
    out["mask_p968_nv868"] = s.make_prefix_mask_np(968, num_valid=868)
    pad = np.zeros(968, np.float32)
    pad[:500] = 1
    pad[600:700] = 1
    out["mask_p968_pad"] = s.make_prefix_mask_np(968, pad_mask=pad)
    out["mask_p968_pad_in"] = pad
    out["time_embs_n10_w1024"] = np.concatenate(s.make_time_embs(10, 1024), 0)
    out["time_embs_n3_w128"] = np.concatenate(s.make_time_embs(3, 128), 0)
    out["sinusoidal_t0.7_w1024"] = ref.openpi_ref.sinusoidal_time_emb(0.7, 1024)
    out["joint_mask_p6_s3"] = ref.openpi_ref.build_joint_additive_mask(6, 3)
    toy_x0 = np.linspace(-1, 1, 24, dtype=np.float32).reshape(1, 4, 6)
    out["euler_x0"] = toy_x0
    out["euler_out"] = s.euler_loop(lambda x, i: np.sin(x + i).astype(np.float32), toy_x0, 5)

    # ---- model pins: oracle (fp32) vs the reference's torch golden (M0, fp32) ----
    for tag, kw in (("mini", recipes.MINI), ("dummy", recipes.DUMMY)):
        cfg = Pi0Config(**{**kw, "dtype": "float32"})
        npar = backbone_named_params(cfg)
        params = O.random_params(npar, seed=0)
        inp = recipes.inputs(cfg, seed=1)
        sd = to_openpi_state_dict(ref, cfg, params)
        import torch

        torch.set_num_threads(os.cpu_count() or 1)
        golden = ref.openpi_ref._SelfContainedRef(cfg, sd, "cpu", torch.float32)
        v_ref = golden.denoise(inp["prefix"], inp["x_t"], inp["time_emb"])
        p32 = O.prepare_params(params, "float32")
        pm = O.prefix_mask(cfg.prefix_len)
        keys, values = O.prefill(p32, cfg, inp["prefix"], pm)
        sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
        v_m1 = O.denoise_step_kv(p32, cfg, keys, values, inp["x_t"], inp["time_emb"], sc, ss, pm)
        v_m0 = O.denoise_step(p32, cfg, inp["prefix"], inp["x_t"], inp["time_emb"])
        for nm, v in (("M1", v_m1), ("M0", v_m0)):
            cos, mx = O.cosine(v, v_ref), O.max_abs(v, v_ref)
            print(f"[golden] {tag} oracle {nm} vs reference _SelfContainedRef: cos={cos:.8f} "
                  f"max_abs={mx:.3e}")
            assert cos >= 0.99999 and mx < 1e-4, (tag, nm, cos, mx)
        out[f"{tag}_v_ref"] = v_ref.astype(np.float32)
        out[f"{tag}_weights_sum"] = np.array(sum(float(np.sum(v, dtype=np.float64))
                                                 for v in params.values()))
        for k, v in inp.items():  # seeded inputs are regenerated; their checksums guard drift
            out[f"{tag}_in_{k}_sum"] = np.array(float(np.sum(v, dtype=np.float64)))

    # ---- dtype-faithful fp16 oracle outputs for the GPU tests (mini) ----
    cfg = Pi0Config(**{**recipes.MINI, "dtype": "float16"})
    params = O.prepare_params(O.random_params(backbone_named_params(cfg), seed=0), "float16")
    inp = recipes.inputs(cfg, seed=1)
    pm = O.prefix_mask(cfg.prefix_len)
    keys, values = O.prefill(params, cfg, inp["prefix"], pm)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    out["mini16_keys"], out["mini16_values"] = keys, values
    out["mini16_v"] = O.denoise_step_kv(params, cfg, keys, values, inp["x_t"], inp["time_emb"],
                                       sc, ss, pm)
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    out["mini16_loop"] = O.denoise_loop_kv(params, cfg, keys, values, inp["noise"], te, sc, ss, pm)

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"[golden] wrote {path} ({os.path.getsize(path) / 1e3:.1f} kB, {len(out)} arrays)")


if __name__ == "__main__":
    main()

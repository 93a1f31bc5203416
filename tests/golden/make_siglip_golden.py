"""Pin the SigLIP oracle to Hugging Face transformers' SigLIP (tests/golden/siglip_golden.npz).

    python tests/golden/make_siglip_golden.py

The reference's vision tower states that it aligns to HF ``SiglipVisionModel`` plus PaliGemma's
``multi_modal_projector`` (``python/mlc_vla/model/pi0/siglip.py:1-10``); the reference itself
needs TVM, which is absent, so its third-party model (``transformers`` 5.5.0 in this image) is
the pin. For each configuration, weights are N(0, 0.02) draws in the vision stage's parameter
order (``oracle.pi0_oracle.random_params``, seed 0) and the image is U(-1, 1) (seed 1); the
weights are loaded into ``SiglipVisionModel`` with the reference loader's layout rules (the
patch-embedding Linear [hidden, p·p·c] is the conv kernel [hidden, c, p, p] permuted to
(p, p, c), ``pi0_loader.py:62``), the model runs in fp32 on channels-first pixels, and the
projector is applied to its ``last_hidden_state``. The oracle's fp32 output must agree to
cosine ≥ 0.99999 before the output is written.

Configurations: ``mini`` (hidden 64, 2 layers, 4 heads, MLP 128, 28×28 image → 4 patches,
projection 32) and ``wide`` (the So400m widths: hidden 1152, MLP 4304, 16 heads of 72, a
224×224 image → 256 patches, projection 2048; one layer so the run stays short).
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
for _p in (REPO, os.path.join(REPO, "mlc-vla_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

PATH = os.path.join(HERE, "siglip_golden.npz")
ROWS = np.arange(0, 256, 16)  # sampled patch rows of the wide configuration


def configs():
    from mlc_vla.model.pi0.pi0_config import Pi0Config, SiglipConfig

    mini = SiglipConfig(image_size=28, patch_size=14, hidden_size=64, intermediate_size=128,
                        num_hidden_layers=2, num_attention_heads=4, projection_dim=32)
    wide = SiglipConfig(num_hidden_layers=1)
    return {"mini": Pi0Config(siglip=mini, dtype="float32"),
            "wide": Pi0Config(siglip=wide, dtype="float32")}


def inputs(cfg, batch=1, seed=1):
    s = cfg.siglip
    rng = np.random.default_rng(seed)
    return rng.uniform(-1.0, 1.0, (batch, s.image_size, s.image_size, s.num_channels)).astype(np.float32)


def hf_forward(cfg, params, image):
    import torch
    from transformers import SiglipVisionConfig, SiglipVisionModel

    s = cfg.siglip
    hc = SiglipVisionConfig(hidden_size=s.hidden_size, intermediate_size=s.intermediate_size,
                            num_hidden_layers=s.num_hidden_layers,
                            num_attention_heads=s.num_attention_heads,
                            num_channels=s.num_channels, image_size=s.image_size,
                            patch_size=s.patch_size, layer_norm_eps=s.layer_norm_eps,
                            hidden_act="gelu_pytorch_tanh")
    model = SiglipVisionModel(hc).eval()
    p = s.patch_size
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32))  # noqa: E731
    sd = {}
    v = "vision_model."
    w = params["vision.patch_embedding.weight"].reshape(s.hidden_size, p, p, s.num_channels)
    sd[v + "embeddings.patch_embedding.weight"] = t(w.transpose(0, 3, 1, 2))
    sd[v + "embeddings.patch_embedding.bias"] = t(params["vision.patch_embedding.bias"])
    sd[v + "embeddings.position_embedding.weight"] = t(params["vision.position_embedding"])
    for i in range(s.num_hidden_layers):
        src, dst = f"vision.layers.{i}.", f"{v}encoder.layers.{i}."
        for name in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                     "self_attn.out_proj", "mlp.fc1", "mlp.fc2", "layer_norm1", "layer_norm2"):
            for leaf in ("weight", "bias"):
                sd[dst + name + "." + leaf] = t(params[src + name + "." + leaf])
    for leaf in ("weight", "bias"):
        sd[v + "post_layernorm." + leaf] = t(params["vision.post_layernorm." + leaf])
    missing, _ = model.load_state_dict(sd, strict=False)
    assert all(k.startswith(v + "head.") for k in missing), missing
    with torch.no_grad():
        hid = model(pixel_values=t(image.transpose(0, 3, 1, 2))).last_hidden_state
        proj = torch.nn.functional.linear(hid, t(params["vision.multi_modal_projector.weight"]),
                                          t(params["vision.multi_modal_projector.bias"]))
    return proj.numpy().astype(np.float32)


def main():
    import torch

    from mlc_vla.model.pi0.pi0_model import vision_named_params
    from oracle import pi0_oracle as O
    from oracle import siglip_oracle as S

    torch.set_num_threads(os.cpu_count() or 1)
    out = {}
    for tag, cfg in configs().items():
        params = O.random_params(vision_named_params(cfg), seed=0)
        image = inputs(cfg, batch=2 if tag == "mini" else 1)
        ref = hf_forward(cfg, params, image)
        mine = S.embed_image(O.prepare_params(params, "float32"), cfg, image)
        cos, mx = O.cosine(mine, ref), O.max_abs(mine, ref)
        print(f"[siglip golden] {tag}: oracle vs transformers SiglipVisionModel: cos={cos:.8f} "
              f"max_abs={mx:.3e}")
        assert cos >= 0.99999, (tag, cos, mx)
        # images are regenerated from their seed by the test; the wide output is kept as 16
        # sampled patch rows plus the L2 norm of every row
        out[f"{tag}_image_sum"] = np.array(float(np.sum(image, dtype=np.float64)))
        if tag == "mini":
            out[f"{tag}_out"] = ref
        else:
            out[f"{tag}_rows"] = ref[:, ROWS]
            out[f"{tag}_row_l2"] = np.sqrt(np.sum(ref.astype(np.float64) ** 2, axis=-1))
    np.savez_compressed(PATH, **out)
    print(f"[siglip golden] wrote {PATH} ({os.path.getsize(PATH) / 1e3:.1f} kB)")


if __name__ == "__main__":
    main()

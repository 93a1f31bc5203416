"""GPU: ``embed_image`` (SigLIP So400m/14 + PaliGemma projector; reference
``python/mlc_vla/model/pi0/siglip.py:20-120``, ``pi0_model.py:97-99``) through ``pi0_embed_image``
against the oracle (``oracle/siglip_oracle.py``, itself pinned to transformers'
``SiglipVisionModel``) on the same seeded weights and images.

Weights are N(0, 0.02²) draws with 1 added to every LayerNorm weight (so normalised activations
stay O(1)); images are U(-1, 1). Tolerances: the kernels and the oracle round at the same places
(matmul accumulate in fp32, one rounding per Linear and per bias add, fp32 LayerNorm, fp32
logits and softmax); the kernels differ in accumulation order, in the fast exponential, and in
rounding the attention probabilities before the final 1/Σ normalisation instead of after it.
"""

import numpy as np
import pytest

from oracle import pi0_oracle as O
from oracle import siglip_oracle as S

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

# (cosine floor, max |Δ| / max |oracle|) per model dtype
TOL = {"float16": (0.99995, 0.01), "bfloat16": (0.9995, 0.03)}


def _config(kind, dtype):
    import dataclasses

    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_config import SiglipConfig

    if kind == "mini":
        s = SiglipConfig(image_size=28, patch_size=14, hidden_size=64, intermediate_size=128,
                         num_hidden_layers=2, num_attention_heads=4, projection_dim=32)
    elif kind == "wide2":  # every So400m width (heads of 72, padded to 80 on the GPU), 2 layers
        s = SiglipConfig(num_hidden_layers=2)
    else:
        s = SiglipConfig()
    return dataclasses.replace(Pi0Config(dtype=dtype), siglip=s)


def _weights(cfg, seed=0):
    from mlc_vla.model.pi0.pi0_model import vision_named_params
    from tests.golden import recipes

    raw = recipes.seeded_weights(vision_named_params(cfg), seed=seed)
    for name, w in raw.items():
        if name.endswith(("layer_norm1.weight", "layer_norm2.weight", "post_layernorm.weight")):
            w += np.float32(1.0)
    return raw


def _images(cfg, n, seed=1):
    s = cfg.siglip
    rng = np.random.default_rng(seed)
    return rng.uniform(-1.0, 1.0, (n, s.image_size, s.image_size, s.num_channels)).astype(np.float32)


class Vision:
    def __init__(self, cfg, max_images):
        from mlc_vla.vision import VisionRuntime

        self.cfg = cfg
        self.raw = _weights(cfg)
        self.rt = VisionRuntime(cfg, device=0, max_images=max_images)
        self.params = self.rt.to_params([self.raw[n] for n, _ in self.rt.named_params])
        self.rt.bind(self.params)

    def run(self, images):
        out = self.rt.embed_image(images)
        torch.cuda.synchronize()
        assert self.rt.device_error() == 0
        return out.float().cpu().numpy()

    def oracle(self, images):
        return S.embed_image(O.prepare_params(self.raw, self.cfg.dtype), self.cfg, images)


def _check(got, want, dtype, what):
    cos = O.cosine(got, want)
    rel = O.max_abs(got, want) / float(np.abs(want).max())
    print(f"[vision] {what}: cos={cos:.6f} max_rel={rel:.3e}")
    lo, hi = TOL[dtype]
    assert np.isfinite(got).all()
    assert cos >= lo and rel <= hi, (what, cos, rel)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("kind,n", [("mini", 2), ("wide2", 3)])
def test_embed_image_matches_oracle(kind, n, dtype):
    cfg = _config(kind, dtype)
    v = Vision(cfg, max_images=n)
    images = _images(cfg, n)
    got = v.run(images)
    s = cfg.siglip
    assert got.shape == (n, s.num_patches, s.projection_dim)
    _check(got, v.oracle(images), dtype, f"{kind} n={n} {dtype}")
    v.rt.close()


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_embed_image_full_so400m_matches_oracle(dtype):
    """All 27 layers at the reference's shapes (224×224×3 -> 256 tokens × 2048)."""
    cfg = _config("full", dtype)
    v = Vision(cfg, max_images=1)
    images = _images(cfg, 1)
    got = v.run(images)
    assert got.shape == (1, 256, 2048)
    _check(got, v.oracle(images), dtype, f"so400m 27 layers {dtype}")
    v.rt.close()


def test_images_of_a_batch_are_independent_and_replay_is_deterministic():
    """Three images in one call equal each image embedded alone (the GEMM tiles differ with the
    row count, the accumulation order per output does not), and a replayed graph reproduces the
    first call bit for bit."""
    cfg = _config("wide2", "float16")
    v = Vision(cfg, max_images=3)
    images = _images(cfg, 3, seed=5)
    x = torch.from_numpy(images).to("cuda", torch.float16)
    out = torch.empty((3, 256, 2048), dtype=torch.float16, device="cuda")
    v.rt.embed_image(x, out=out)
    first = out.clone()
    launches = v.rt.launch_count()
    v.rt.embed_image(x, out=out)  # same pointers: the cached graph replays
    torch.cuda.synchronize()
    assert torch.equal(out, first)
    assert v.rt.launch_count() - launches == launches  # one call's kernels, counted per replay
    for i in range(3):
        alone = v.rt.embed_image(x[i:i + 1].contiguous())
        torch.cuda.synchronize()
        d = (alone[0].float() - first[i].float()).abs().max().item()
        assert d <= 2e-3 * first[i].float().abs().max().item(), (i, d)
    v.rt.close()


def test_vm_style_call_and_argument_errors():
    from mlc_vla import _lib

    cfg = _config("mini", "float16")
    v = Vision(cfg, max_images=2)
    images = _images(cfg, 2)
    got = v.rt["embed_image"](images, v.params).numpy()
    assert got.shape == (2, 4, 32)
    with pytest.raises(ValueError, match="max_images"):
        v.rt.embed_image(_images(cfg, 3))
    lib = _lib.load()
    stream = v.rt._stream()
    x = torch.zeros((1, 28, 28, 3), dtype=torch.float16, device="cuda")
    out = torch.empty((1, 4, 32), dtype=torch.float16, device="cuda")
    assert lib.pi0_embed_image(v.rt._ctx, 0, x.data_ptr(), out.data_ptr(), stream) == _lib.PI0_ERR_INVALID
    assert lib.pi0_embed_image(v.rt._ctx, 1, None, out.data_ptr(), stream) == _lib.PI0_ERR_INVALID
    from mlc_vla.vision import VisionRuntime

    fresh = VisionRuntime(cfg, device=0, max_images=1)
    assert lib.pi0_embed_image(fresh._ctx, 1, x.data_ptr(), out.data_ptr(), stream) == _lib.PI0_ERR_NO_PARAMS
    fresh.close()
    v.rt.close()

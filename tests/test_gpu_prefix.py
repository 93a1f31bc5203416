"""GPU: prefix assembly (the reference assembles ``prefix_embs`` on the host from
``embed_image`` / ``embed_language``, ``python/mlc_vla/sample.py:11-13``; layout
``pi0_config.py:126-131``): image tokens and language embeddings written in place into one
prefix buffer by ``mlc_vla.prefix.assemble_prefix``, equal bit for bit to the separately computed
pieces concatenated, within tolerance of the oracles' pieces, with openpi's pad bits, and fed to
``prefill``."""

import dataclasses

import numpy as np
import pytest

from oracle import pi0_oracle as O
from oracle import siglip_oracle as S

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _config():
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_config import SiglipConfig
    from tests.golden import recipes

    base = Pi0Config(**{**recipes.MINI, "dtype": "float16"})
    sig = SiglipConfig(image_size=56, patch_size=14, hidden_size=64, intermediate_size=128,
                       num_hidden_layers=2, num_attention_heads=4,
                       projection_dim=base.vlm.width)
    return dataclasses.replace(base, image_keys=("base_0_rgb", "left_wrist_0_rgb"), siglip=sig,
                               max_token_len=24)


def test_prefix_assembled_in_place_equals_pieces_and_oracle():
    from mlc_vla.model.pi0.pi0_model import vision_named_params
    from mlc_vla.prefix import assemble_prefix, prefix_pad_bits
    from mlc_vla.runtime import embed_language
    from mlc_vla.vision import VisionRuntime
    from tests.golden import recipes

    cfg = _config()
    s = cfg.siglip
    assert cfg.prefix_len == 2 * 16 + 24
    raw = recipes.seeded_weights(vision_named_params(cfg), seed=3)
    for n, w in raw.items():
        if n.endswith(("layer_norm1.weight", "layer_norm2.weight", "post_layernorm.weight")):
            w += np.float32(1.0)
    vis = VisionRuntime(cfg, device=0, max_images=2)
    vis.bind(vis.to_params([raw[n] for n, _ in vis.named_params]))
    rng = np.random.default_rng(7)
    B, vocab, W = 2, 500, cfg.vlm.width
    images = rng.uniform(-1, 1, (B, 2, 56, 56, 3)).astype(np.float32)
    ids = rng.integers(0, vocab, size=(B, 24)).astype(np.int32)
    table_np = (0.02 * rng.standard_normal((vocab, W))).astype(np.float32)
    table = torch.from_numpy(table_np).to("cuda", torch.float16)
    image_masks = np.array([[1, 0], [1, 1]], np.float32)
    token_mask = np.zeros((B, 24), np.float32)
    token_mask[0, :10] = 1
    token_mask[1, :24] = 1

    prefix, pad = assemble_prefix(vis, table, images, ids, image_masks, token_mask)
    torch.cuda.synchronize()
    assert prefix.shape == (B, cfg.prefix_len, W) and prefix.dtype == torch.float16
    assert pad.shape == (B, cfg.prefix_len)
    assert pad[0, :16].all() and not pad[0, 16:32].any() and pad[0, 32:42].all()
    assert not pad[0, 42:].any() and pad[1].all()
    np.testing.assert_array_equal(pad, prefix_pad_bits(cfg, image_masks, token_mask, B))

    for b in range(B):
        img = vis.embed_image(images[b])
        lang = embed_language(table, ids[b])
        torch.cuda.synchronize()
        want = torch.cat([img.reshape(-1, W), lang.reshape(-1, W)], 0)
        assert torch.equal(prefix[b], want)
        # the pieces against the oracles
        p = O.prepare_params(raw, "float16")
        oi = S.embed_image(p, cfg, images[b]).reshape(-1, W)
        ol = np.asarray(O.embed_language(table_np, ids[b], "float16"), np.float32).reshape(-1, W)
        got = prefix[b].float().cpu().numpy()
        assert O.cosine(got[:32], oi) >= 0.99995
        assert np.array_equal(got[32:], ol)
    vis.close()


def test_assembled_prefix_feeds_prefill_with_its_pad_mask():
    """prefill on the GPU-assembled prefix equals prefill on the same prefix staged from the host,
    and padded keys carry no weight: changing a padded row's embedding leaves every valid row's
    K/V unchanged."""
    from mlc_vla.model.pi0.pi0_model import backbone_named_params, vision_named_params
    from mlc_vla.prefix import assemble_prefix
    from mlc_vla.runtime import Pi0Runtime
    from mlc_vla.sample import make_prefix_mask_np
    from mlc_vla.vision import VisionRuntime
    from tests.golden import recipes

    cfg = _config()
    raw = recipes.seeded_weights(vision_named_params(cfg), seed=4)
    vis = VisionRuntime(cfg, device=0, max_images=2)
    vis.bind(vis.to_params([raw[n] for n, _ in vis.named_params]))
    rt = Pi0Runtime(cfg, device=0)
    rt.bind(rt.to_params([v for v in O.random_params(backbone_named_params(cfg), seed=0).values()]))
    rng = np.random.default_rng(9)
    images = rng.uniform(-1, 1, (2, 56, 56, 3)).astype(np.float32)
    ids = rng.integers(0, 300, size=(24,)).astype(np.int32)
    table = (0.02 * torch.randn((300, cfg.vlm.width), device="cuda")).half()
    tm = np.zeros(24, np.float32)
    tm[:15] = 1
    prefix, pad = assemble_prefix(vis, table, images, ids, token_mask=tm)
    mask = make_prefix_mask_np(cfg.prefix_len, pad_mask=pad[0])
    k1, v1 = rt.prefill(prefix, mask)
    host = prefix.cpu()
    k2, v2 = rt.prefill(host, mask)
    torch.cuda.synchronize()
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
    changed = prefix.clone()
    changed[0, -1] += 1.0  # a padded language row
    k3, v3 = rt.prefill(changed, mask)
    torch.cuda.synchronize()
    valid = torch.from_numpy(pad[0] > 0).cuda()
    assert torch.equal(k1[:, :, :, valid], k3[:, :, :, valid])
    assert torch.equal(v1[:, :, :, valid], v3[:, :, :, valid])
    vis.close()
    rt.close()

"""CPU oracle for ``embed_image`` (SigLIP So400m/14 + PaliGemma projector) — TEST
INFRASTRUCTURE, NOT PRODUCT CODE.

Only ``tests/`` may import this module, as the checker; the product path (``mlc_vla`` +
``libpi0b200.so``) never calls it.

A numpy restatement of the reference's vision tower with its dtype placement made explicit (the
conventions of ``pi0_oracle``: a model-dtype matmul accumulates in fp32 and rounds once, a bias
add rounds again, GELU-tanh is evaluated in fp32 and rounded once):

* ``python/mlc_vla/model/pi0/siglip.py:104-120``  patchify (channels-last, non-overlapping
  p × p patches flattened in (row, column, channel) order), patch-embedding Linear, + position
  embedding, the encoder layers, post LayerNorm, multi-modal projector;
* ``siglip.py:23-37``   LayerNorm computed in fp32 (mean, biased variance, eps) then cast;
* ``siglip.py:50-72``   attention: q·scale in the model dtype, logits from fp32 q and k, fp32
  softmax, probabilities in the model dtype, context = probs · v (model-dtype output);
* ``siglip.py:40-47``   MLP: fc2(gelu_tanh(fc1(x)));
* ``siglip.py:78-88``   pre-norm residual blocks.

Pinning: ``tests/golden/make_siglip_golden.py`` runs Hugging Face ``transformers``'
``SiglipVisionModel`` (the implementation the reference states it aligns to, ``siglip.py:3``;
transformers 5.5 in this image) with the same weights in fp32 and commits its outputs;
``tests/test_siglip_oracle.py`` requires this oracle to match them.
"""

from __future__ import annotations

import numpy as np

from .pi0_oracle import F32, gelu_tanh, linear, rnd


def patchify(image, patch: int) -> np.ndarray:
    """``siglip.py:104-114``: [B, H, W, C] -> [B, (H/p)·(W/p), p·p·C]."""
    image = np.asarray(image, F32)
    b, hgt, wid, c = image.shape
    sh, sw = hgt // patch, wid // patch
    x = image.reshape(b, sh, patch, sw, patch, c).transpose(0, 1, 3, 2, 4, 5)
    return x.reshape(b, sh * sw, patch * patch * c)


def layer_norm(x, w, b, eps, dt):
    """``siglip.py:23-37``: fp32 LayerNorm (biased variance), then the model dtype."""
    x = np.asarray(x, F32)
    d = F32(x.shape[-1])
    mean = np.sum(x, axis=-1, keepdims=True, dtype=F32) / d
    xc = x - mean
    var = np.sum(xc * xc, axis=-1, keepdims=True, dtype=F32) / d
    return rnd(xc / np.sqrt(var + F32(eps)) * w + b, dt)


def attention(p, pre, x, heads, dt):
    """``siglip.py:50-72`` for x [B, T, hidden] (model dtype)."""
    b, t, hid = x.shape
    hd = hid // heads
    # ``q * self.scale`` (siglip.py:65): the Relax nn frontend turns a Python scalar operand into
    # a constant of the tensor's dtype, so the scale itself is rounded to the model dtype
    scale = rnd(F32(hd ** -0.5), dt)

    def proj(name):
        y = linear(x, p[pre + name + ".weight"], p[pre + name + ".bias"], dt)
        return y.reshape(b, t, heads, hd).transpose(0, 2, 1, 3)

    q, k, v = proj("q_proj"), proj("k_proj"), proj("v_proj")
    qs = rnd(q * scale, dt)
    logits = np.matmul(qs, np.swapaxes(k, -1, -2)).astype(F32)
    m = np.max(logits, axis=-1, keepdims=True)
    e = np.exp(logits - m)
    probs = rnd(e / np.sum(e, axis=-1, keepdims=True, dtype=F32), dt)
    ctx = rnd(np.matmul(probs, v), dt)
    ctx = ctx.transpose(0, 2, 1, 3).reshape(b, t, hid)
    return linear(ctx, p[pre + "out_proj.weight"], p[pre + "out_proj.bias"], dt)


def mlp(p, pre, x, dt):
    h = linear(x, p[pre + "fc1.weight"], p[pre + "fc1.bias"], dt)
    h = rnd(gelu_tanh(h), dt)
    return linear(h, p[pre + "fc2.weight"], p[pre + "fc2.bias"], dt)


def embed_image(p, cfg, image) -> np.ndarray:
    """``Pi0Model.embed_image`` (``pi0_model.py:97-99``): image [B, H, W, C] (any float dtype)
    -> [B, num_patches, projection_dim] in the model dtype (held as fp32)."""
    s = cfg.siglip
    dt = cfg.dtype
    eps = s.layer_norm_eps
    x = rnd(patchify(rnd(image, dt), s.patch_size), dt)
    x = linear(x, p["vision.patch_embedding.weight"], p["vision.patch_embedding.bias"], dt)
    x = rnd(x + p["vision.position_embedding"][None], dt)
    for i in range(s.num_hidden_layers):
        pre = f"vision.layers.{i}."
        a = attention(p, pre + "self_attn.", layer_norm(x, p[pre + "layer_norm1.weight"],
                                                         p[pre + "layer_norm1.bias"], eps, dt),
                      s.num_attention_heads, dt)
        x = rnd(x + a, dt)
        m = mlp(p, pre + "mlp.", layer_norm(x, p[pre + "layer_norm2.weight"],
                                            p[pre + "layer_norm2.bias"], eps, dt), dt)
        x = rnd(x + m, dt)
    x = layer_norm(x, p["vision.post_layernorm.weight"], p["vision.post_layernorm.bias"], eps, dt)
    return linear(x, p["vision.multi_modal_projector.weight"],
                  p["vision.multi_modal_projector.bias"], dt)

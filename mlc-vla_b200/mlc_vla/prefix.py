"""Prefix assembly on the GPU: image tokens and language embeddings written in place into one
``prefix_embs`` buffer, plus the pad bits that ``PiZeroRunner.sample(prefix_pad=…)`` takes.

The reference assembles the prefix on the host from its ``embed_image`` / ``embed_language``
outputs (``python/mlc_vla/sample.py:11-13``): ``prefix_len = num_images · num_patches +
max_token_len`` (``pi0_config.py:126-131``), the images in ``image_keys`` order, then the
language tokens; ``prefix_pad`` holds openpi's prefix pad masks (an image's mask repeated over
its patches, then the token mask), from which ``make_prefix_mask_np`` builds the additive mask
(``sample.py:50-64``). Here both embedding kernels write straight into their rows of the
prefix buffer (``pi0_embed_image`` into rows ``[i·T, (i+1)·T)`` of each request, then
``pi0_embed_language`` into the ``max_token_len`` rows after the images), so the assembly costs
no copy; padded rows keep their embeddings and are hidden by the mask, as in the reference.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from .runtime import TORCH_DTYPE, embed_language, to_device


def prefix_pad_bits(config, image_masks=None, token_mask=None, batch: int = 1) -> np.ndarray:
    """[batch, prefix_len] float32 0/1 valid bits: each image's mask over its num_patches rows,
    then the token mask (all valid when a mask is None)."""
    n_img, T, L = config.num_images, config.siglip.num_patches, config.max_token_len
    im = np.ones((batch, n_img), np.float32) if image_masks is None else \
        np.asarray(image_masks, np.float32).reshape(batch, n_img)
    tm = np.ones((batch, L), np.float32) if token_mask is None else \
        np.asarray(token_mask, np.float32).reshape(batch, L)
    return np.concatenate([np.repeat(im, T, axis=1), tm], axis=1)


def assemble_prefix(vision, table: torch.Tensor, images, token_ids, image_masks=None,
                    token_mask=None, out: Optional[torch.Tensor] = None):
    """prefix_embs [B, prefix_len, width] (model dtype, on the vision runtime's GPU) and
    prefix_pad [B, prefix_len] (host float32 0/1) for B requests.

    vision: a ``VisionRuntime`` with bound parameters (its projection_dim = the prefix expert's
    width); table: the prefix expert's token embedding [vocab, width] on the same GPU; images
    [B, num_images, S, S, C] (or [num_images, S, S, C] for B = 1); token_ids [B, max_token_len]
    int (or [max_token_len])."""
    cfg = vision.config
    s = cfg.siglip
    n_img, T, L = cfg.num_images, s.num_patches, cfg.max_token_len
    P, W = cfg.prefix_len, s.projection_dim
    if table.shape[1] != W:
        raise ValueError(f"embedding width {table.shape[1]} != projection_dim {W}")
    dev = vision.device
    x = to_device(images, vision.dtype, dev).reshape(-1, n_img, s.image_size, s.image_size,
                                                     s.num_channels)
    B = x.shape[0]
    ids = torch.as_tensor(np.asarray(token_ids) if not isinstance(token_ids, torch.Tensor)
                          else token_ids).reshape(B, L)
    if out is None:
        out = torch.empty((B, P, W), dtype=TORCH_DTYPE[vision.dtype], device=dev)
    elif tuple(out.shape) != (B, P, W) or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous ({B}, {P}, {W}) tensor")
    for b in range(B):
        if n_img:
            vision.embed_image(x[b], out=out[b, : n_img * T].view(n_img, T, W))
        embed_language(table, ids[b], out=out[b, n_img * T:])
    return out, prefix_pad_bits(cfg, image_masks, token_mask, B)

"""CPU: the prefix layout and pad bits of ``mlc_vla.prefix`` (``pi0_config.py:126-131``: images
in ``image_keys`` order, num_patches rows each, then max_token_len language rows)."""

import numpy as np


def test_prefix_pad_bits_layout():
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.prefix import prefix_pad_bits

    cfg = Pi0Config()
    assert cfg.prefix_len == 3 * 256 + 200
    pad = prefix_pad_bits(cfg, image_masks=[1, 0, 1], token_mask=np.r_[np.ones(37), np.zeros(163)])
    assert pad.shape == (1, 968) and pad.dtype == np.float32
    assert pad[0, :256].all() and not pad[0, 256:512].any() and pad[0, 512:768].all()
    assert pad[0, 768:805].all() and not pad[0, 805:].any()
    assert prefix_pad_bits(cfg, batch=2).shape == (2, 968)
    assert prefix_pad_bits(cfg).all()

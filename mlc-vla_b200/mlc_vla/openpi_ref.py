"""Host-side input helpers shared with openpi (no model code).

``sinusoidal_time_emb`` restates openpi's ``create_sinusoidal_pos_embedding`` as the reference
does (``python/mlc_vla/openpi_ref.py:49-58``): min period 4e-3, max period 4.0, computed in
float64, returned as [1, dim] fp32 ``concat(sin, cos)``. ``build_joint_additive_mask`` is the
π0.5 joint mask of the M0 path (``openpi_ref.py:61-69``).
"""

from __future__ import annotations

import math

import numpy as np

_ATTN_NEG_INF = -2.3819763e38


def sinusoidal_time_emb(timestep: float, dim: int) -> np.ndarray:
    if dim % 2 != 0:
        raise ValueError("dim must be even")
    time = np.array([timestep], dtype=np.float64)
    fraction = np.linspace(0.0, 1.0, dim // 2, dtype=np.float64)
    period = 4e-3 * (4.0 / 4e-3) ** fraction
    scaling = 1.0 / period * 2 * math.pi
    sin_in = scaling[None, :] * time[:, None]
    return np.concatenate([np.sin(sin_in), np.cos(sin_in)], axis=1).astype(np.float32)


def build_joint_additive_mask(prefix_len: int, suffix_len: int) -> np.ndarray:
    total = prefix_len + suffix_len
    att = np.zeros(total, dtype=np.int32)
    att[prefix_len] = 1
    cumsum = np.cumsum(att)
    allow = cumsum[None, :] <= cumsum[:, None]
    mask = np.where(allow, 0.0, _ATTN_NEG_INF).astype(np.float32)
    return mask.reshape(1, 1, total, total)

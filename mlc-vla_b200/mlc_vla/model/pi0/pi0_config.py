"""π0.5 configuration: the shape contract of the M1 hot path.

Field names, defaults and derived sizes follow the reference configuration
(``python/mlc_vla/model/pi0/pi0_config.py:17-170``) so that callers which build a
``Pi0Config`` for the reference build the same object here:

* ``GemmaExpertConfig.from_variant`` knows ``gemma_2b`` (prefix / PaliGemma expert),
  ``gemma_300m`` (action expert) and ``dummy`` exactly as the reference does
  (``pi0_config.py:31-44``). Two more variants, ``mini_vlm`` and ``mini_action``, give the
  small dual-expert model that the CPU-runnable benchmark configuration describes
  (prefix width 256 / 2 layers / 4 heads / head_dim 64 / GeGLU 1024; action width 128 /
  GeGLU 512); ``gemma_2b_2l`` / ``gemma_300m_2l`` keep every π0.5 width with 2 layers, for
  parity runs at full width that a CPU oracle finishes in seconds.
* ``prefix_len = num_images * num_patches + max_token_len`` and ``suffix_len =
  action_horizon`` (``pi0_config.py:129-136``).
* ``from_openpi_config`` reads ``action_dim``, ``action_horizon`` and the two variant names
  from an openpi ``config.json`` and applies keyword overrides (``pi0_config.py:142-163``).
* The two experts must agree on ``head_dim``, ``num_heads``, ``num_kv_heads`` and
  ``depth``; a mismatch raises ``AssertionError`` at construction
  (``pi0_config.py:165-170``), because both experts share one attention.
"""

from __future__ import annotations

import dataclasses
import json
import os
from typing import Dict, List, Tuple

# name -> (width, depth, mlp_dim, num_heads, num_kv_heads, head_dim)
_VARIANTS: Dict[str, Tuple[int, int, int, int, int, int]] = {
    "gemma_2b": (2048, 18, 16_384, 8, 1, 256),
    "gemma_300m": (1024, 18, 4096, 8, 1, 256),
    "dummy": (64, 4, 128, 8, 1, 16),
    "mini_vlm": (256, 2, 1024, 4, 1, 64),
    "mini_action": (128, 2, 512, 4, 1, 64),
    "gemma_2b_2l": (2048, 2, 16_384, 8, 1, 256),
    "gemma_300m_2l": (1024, 2, 4096, 8, 1, 256),
}


@dataclasses.dataclass
class GemmaExpertConfig:
    """One Gemma expert (prefix / PaliGemma expert or action expert)."""

    width: int
    depth: int
    mlp_dim: int
    num_heads: int
    num_kv_heads: int
    head_dim: int

    @staticmethod
    def from_variant(variant: str) -> "GemmaExpertConfig":
        if variant not in _VARIANTS:
            raise ValueError(f"Unknown gemma variant: {variant}")
        return GemmaExpertConfig(*_VARIANTS[variant])


@dataclasses.dataclass
class SiglipConfig:
    """SigLIP So400m/14 vision tower sizes; only ``num_patches`` feeds the prefix length."""

    image_size: int = 224
    patch_size: int = 14
    num_channels: int = 3
    hidden_size: int = 1152
    intermediate_size: int = 4304
    num_hidden_layers: int = 27
    num_attention_heads: int = 16
    layer_norm_eps: float = 1e-6
    projection_dim: int = 2048

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def num_patches(self) -> int:
        side = self.image_size // self.patch_size
        return side * side


@dataclasses.dataclass
class Pi0Config:
    """Top-level π0.5 configuration (defaults: the LIBERO π0.5 checkpoint)."""

    paligemma_variant: str = "gemma_2b"
    action_expert_variant: str = "gemma_300m"
    action_dim: int = 32
    action_horizon: int = 10
    max_token_len: int = 200
    pi05: bool = True
    siglip: SiglipConfig = dataclasses.field(default_factory=SiglipConfig)
    image_keys: Tuple[str, ...] = ("base_0_rgb", "left_wrist_0_rgb", "right_wrist_0_rgb")
    dtype: str = "float32"
    attn_logits_dtype: str = "float32"
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10_000.0
    attn_neg_inf: float = -2.3819763e38
    time_min_period: float = 4e-3
    time_max_period: float = 4.0
    num_denoise_steps: int = 10
    kwargs: Dict[str, object] = dataclasses.field(default_factory=dict)

    @property
    def vlm(self) -> GemmaExpertConfig:
        return GemmaExpertConfig.from_variant(self.paligemma_variant)

    @property
    def action_expert(self) -> GemmaExpertConfig:
        return GemmaExpertConfig.from_variant(self.action_expert_variant)

    @property
    def num_images(self) -> int:
        return len(self.image_keys)

    @property
    def prefix_len(self) -> int:
        return self.num_images * self.siglip.num_patches + self.max_token_len

    @property
    def suffix_len(self) -> int:
        return self.action_horizon

    def experts(self) -> List[GemmaExpertConfig]:
        return [self.vlm, self.action_expert]

    @classmethod
    def from_openpi_config(cls, path: str, **overrides) -> "Pi0Config":
        if os.path.isdir(path):
            path = os.path.join(path, "config.json")
        with open(path) as f:
            raw = json.load(f)
        kwargs: Dict[str, object] = {
            k: raw[k]
            for k in ("action_dim", "action_horizon", "paligemma_variant", "action_expert_variant")
            if k in raw
        }
        kwargs.update(overrides)
        return cls(**kwargs)

    def __post_init__(self):
        a, b = self.vlm, self.action_expert
        assert a.head_dim == b.head_dim, "experts must share head_dim"
        assert a.num_heads == b.num_heads, "experts must share num_heads"
        assert a.num_kv_heads == b.num_kv_heads, "experts must share num_kv_heads"
        assert a.depth == b.depth, "experts must share depth"

"""Helpers shared by the comparison harnesses (compare_kv, compare_loop, compare_pad,
compare_quant): cosine, seeded random weights in parameter-table order, and the M1 call
sequence. They use only this package's public functions, like the reference's harnesses."""

from __future__ import annotations

import dataclasses
from typing import Dict, List

import numpy as np


def on_device_dtype(config):
    """The library computes in fp16 or bf16: an fp32 configuration (the reference harnesses'
    CPU default) runs in fp16."""
    if config.dtype in ("float16", "bfloat16"):
        return config
    return dataclasses.replace(config, dtype="float16")


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-12))


def max_abs(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def random_weights(named_params, rng: np.random.Generator) -> Dict[str, np.ndarray]:
    """N(0, 0.02) float weights (zeros for integer entries), fp32, keyed by parameter name."""
    out = {}
    for name, p in named_params:
        shape = [int(s) for s in p.shape]
        if p.dtype.startswith(("int", "uint")):
            out[name] = np.zeros(shape, p.dtype)
        else:
            out[name] = (0.02 * rng.standard_normal(shape)).astype(np.float32)
    return out


def in_order(named_params, weights: Dict[str, np.ndarray]) -> List[np.ndarray]:
    return [weights[n] for n, _ in named_params]


def m1_step(ex, params, config, prefix, x_t, time_emb, num_valid: int):
    """prefill + denoise_step_kv through the VM-style interface, fp32 v_t on the host."""
    from mlc_vla.sample import make_prefix_mask_np, make_rope_np

    pmask = make_prefix_mask_np(config.prefix_len, num_valid=num_valid)
    cos, sin = make_rope_np(config.suffix_len, config.vlm.head_dim, config.rope_theta,
                            offset=num_valid)
    keys, values = ex["prefill"](prefix, pmask, params)
    return ex["denoise_step_kv"](keys, values, x_t, time_emb, cos, sin, pmask, params).numpy()

"""CPU oracle for group quantisation — TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may use it, as the
checker for the GPU quantiser and the dequant-in-load-path kernels.

Restates the vendored mlc-llm group quantiser of the reference
(``python/mlc_vla/quant.py``), NK layout, quantisation along K (``quant.py:148,158-164``):

* ``_quantize`` (``quant.py:217-266``): per group of ``G`` elements along K,
  ``max_abs = max |w|`` in the model dtype (padding lanes excluded); ``scale = max_abs /
  max_int`` rounded to the model dtype; ``code = clamp(round(w/scale + max_int), 0,
  2·max_int)`` where each arithmetic op rounds to the model dtype; codes become uint32.
* ``pack_weight`` (``quant.py:65-86``): element r of storage word j sits at bit
  ``r·bits``; lanes past K are 0.
* ``convert_uint_to_float`` + ``_dequantize`` (``quant.py:46-62,176-193``):
  ``w = (float(code) − max_int)·scale`` in the model dtype.

``round`` is TVM's ``tir.round``, which the LLVM backend lowers to ``llvm.round`` (round
half away from zero); ``max(NaN, 0)`` takes the 0 branch (select semantics), so an
all-zero group (scale 0, 0/0) yields code 0. Parity of this restatement is UNPINNED against
an executed reference: the reference quantiser needs TVM, which is not installed, and the
reference ships no quantised fixtures.
"""

from __future__ import annotations

import numpy as np

from .pi0_oracle import rnd

F32 = np.float32

# name -> (group_size, bits, elems_per_uint32, max_int, model_dtype)
PRESETS = {
    "q4f16_1": (32, 4, 8, 7, "float16"),
    "q4bf16_1": (32, 4, 8, 7, "bfloat16"),
    "q3f16_1": (40, 3, 10, 3, "float16"),
}


def _round_half_away(x):
    return (np.sign(x) * np.floor(np.abs(x) + F32(0.5))).astype(F32)


def quantize(w: np.ndarray, preset: str):
    """w [N, K] (model-dtype values) → (q_weight [N, ng·G/epw] uint32, q_scale [N, ng] fp32
    holding model-dtype values)."""
    g, bits, epw, maxint, dt = PRESETS[preset]
    w = rnd(np.asarray(w, F32), dt)
    n, k = w.shape
    ng = -(-k // g)
    kp = ng * g
    wp = np.zeros((n, kp), F32)
    wp[:, :k] = w
    a = np.abs(wp)
    a[:, k:] = -np.inf
    max_abs = a.reshape(n, ng, g).max(axis=-1)
    with np.errstate(divide="ignore", invalid="ignore"):
        scale = rnd(max_abs / F32(maxint), dt)
        s_full = np.repeat(scale, g, axis=1)
        t = rnd(wp / s_full, dt)
        t = rnd(t + F32(maxint), dt)
    t = _round_half_away(t)
    t = np.where(t > 0, t, F32(0))          # max(t, 0) with select semantics (NaN → 0)
    t = np.where(t < 2 * maxint, t, F32(2 * maxint))
    codes = t.astype(np.uint32)
    codes[:, k:] = 0
    words = codes.reshape(n, kp // epw, epw)
    shifts = (np.arange(epw, dtype=np.uint32) * bits)[None, None, :]
    packed = np.bitwise_or.reduce(words << shifts, axis=-1).astype(np.uint32)
    return packed, scale


def unpack_codes(q_weight: np.ndarray, preset: str, k: int) -> np.ndarray:
    """uint32 words → codes [N, K]."""
    g, bits, epw, maxint, dt = PRESETS[preset]
    n, nw = q_weight.shape
    shifts = (np.arange(epw, dtype=np.uint32) * bits)[None, None, :]
    codes = (q_weight[:, :, None] >> shifts) & np.uint32((1 << bits) - 1)
    return codes.reshape(n, nw * epw)[:, :k]


def dequantize(q_weight: np.ndarray, q_scale: np.ndarray, preset: str, k: int) -> np.ndarray:
    """(code − max_int)·scale in the model dtype → [N, K] fp32 holding model-dtype values."""
    g, bits, epw, maxint, dt = PRESETS[preset]
    codes = unpack_codes(q_weight, preset, k).astype(F32)
    s = np.repeat(np.asarray(q_scale, F32), g, axis=1)[:, :k]
    return rnd((codes - F32(maxint)) * s, dt)

"""CPU: group-quantisation oracle — known answers from the format definition
(python/mlc_vla/quant.py:46-86,176-266) and its size-independent properties."""

import numpy as np
import pytest

from oracle import quant_oracle as Q


def test_q4_known_answer():
    # one group of 32: max|w| = 0.7 -> scale = fp16(0.7/7) = fp16(0.1)
    w = np.zeros((1, 32), np.float32)
    w[0, :8] = [0.7, -0.7, 0.0, 0.35, -0.35, 0.1, 0.05, -0.049]
    q, s = Q.quantize(w, "q4f16_1")
    s16 = np.float16(np.float16(0.7) / np.float16(7.0))
    assert s[0, 0] == np.float32(s16)
    codes = Q.unpack_codes(q, "q4f16_1", 32)[0]
    # w/s + 7 in fp16 -> round half away from zero -> clamp [0, 14]
    exp = []
    for x in w[0]:
        t = np.float16(np.float16(np.float16(x) / s16) + np.float16(7))
        exp.append(int(np.clip(np.sign(t) * np.floor(abs(float(t)) + 0.5), 0, 14)))
    assert list(codes) == exp
    assert codes[0] == 14 and codes[1] == 0 and codes[2] == 7
    # packing: element r at bit 4r, LSB first
    assert q.shape == (1, 4) and q.dtype == np.uint32
    assert (int(q[0, 0]) & 0xF) == codes[0] and ((int(q[0, 0]) >> 4) & 0xF) == codes[1]


def test_q3_partial_group_and_packing():
    rng = np.random.default_rng(0)
    w = (0.02 * rng.standard_normal((3, 50))).astype(np.float32)  # 2 groups of 40, tail of 10
    q, s = Q.quantize(w, "q3f16_1")
    assert q.shape == (3, 8) and s.shape == (3, 2)
    codes = Q.unpack_codes(q, "q3f16_1", 80)
    assert np.all(codes[:, 50:] == 0)          # lanes past K pack as 0
    assert np.all(codes <= 6)
    assert np.all((q >> np.uint32(30)) == 0)   # 10 codes × 3 bits use bits 0..29
    # tail group's scale comes from the 10 valid elements only
    t = np.abs(w[:, 40:50].astype(np.float16).astype(np.float32)).max(axis=1)
    assert np.array_equal(s[:, 1], (t / np.float32(3)).astype(np.float16).astype(np.float32))


@pytest.mark.parametrize("preset", ["q4f16_1", "q4bf16_1", "q3f16_1"])
def test_dequant_error_bounded_by_half_step(preset):
    rng = np.random.default_rng(1)
    w = (0.02 * rng.standard_normal((64, 200))).astype(np.float32)
    q, s = Q.quantize(w, preset)
    dq = Q.dequantize(q, s, preset, 200)
    g = Q.PRESETS[preset][0]
    step = np.repeat(s, g, axis=1)[:, :200]
    wd = Q.rnd(w, Q.PRESETS[preset][4])
    # bf16 keeps 8 significand bits, so w/s and w/s + max_int round coarser than fp16
    slack = 0.6 if preset == "q4bf16_1" else 0.51
    assert np.all(np.abs(dq - wd) <= slack * step + 2.0 ** -8 * np.abs(wd) + 1e-8)


def test_all_zero_group_gives_code_zero():
    q, s = Q.quantize(np.zeros((1, 32), np.float32), "q4f16_1")
    assert s[0, 0] == 0 and q[0, 0] == 0 and q.sum() == 0
    assert np.all(Q.dequantize(q, s, "q4f16_1", 32) == 0)

"""GPU parity: libpi0b200 (through its C ABI) against the CPU oracle and the committed fixtures.

Tolerances (the hot-path contract): end outputs cosine ≥ 0.9995 and max-abs ≤ 2e-2 in fp16;
fp32 K cache within 1e-2 relative of the oracle's; bit-exact where the math is identical by
construction (in-graph loop vs host-stepped loop).
"""

import numpy as np
import pytest
import torch

from conftest import cosine, max_abs
from gpu_common import Model, config
from oracle import pi0_oracle as O
from tests.golden import recipes

pytestmark = pytest.mark.gpu

COS, MAXABS = 0.9995, 2e-2


def _np(t):
    return t.float().cpu().numpy()


@pytest.fixture(scope="module")
def mini():
    return Model(config(recipes.MINI), max_batch=4)


def _check(out, ref, cos=COS, mx=MAXABS, what=""):
    c, m = cosine(out, ref), max_abs(out, ref)
    print(f"[parity] {what}: cos={c:.7f} max_abs={m:.3e}")
    assert c >= cos and m <= mx, (what, c, m)


def test_prefill_kv_matches_golden(mini, golden):
    inp = mini.inputs()
    pm = O.prefix_mask(mini.cfg.prefix_len)
    k, v = mini.rt.prefill(inp["prefix"], pm)
    torch.cuda.synchronize()
    kr, vr = golden["mini16_keys"], golden["mini16_values"]
    assert k.shape == kr.shape and k.dtype == torch.float32 and v.dtype == torch.float16
    _check(_np(k), kr, 0.99999, 1e-2 * np.abs(kr).max(), "prefill keys")
    _check(_np(v), vr, 0.99999, 1e-2 * np.abs(vr).max(), "prefill values")


def test_denoise_step_kv_matches_golden(mini, golden):
    inp = mini.inputs()
    cfg = mini.cfg
    pm = O.prefix_mask(cfg.prefix_len)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    # oracle K/V in (isolates the step), then the full GPU chain
    v1 = mini.rt.denoise_step_kv(golden["mini16_keys"], golden["mini16_values"], inp["x_t"],
                                 inp["time_emb"], sc, ss, pm)
    _check(_np(v1), golden["mini16_v"], what="step on oracle K/V")
    k, vv = mini.rt.prefill(inp["prefix"], pm)
    v2 = mini.rt.denoise_step_kv(k, vv, inp["x_t"], inp["time_emb"], sc, ss, pm)
    assert v2.dtype == torch.float32 and tuple(v2.shape) == (1, cfg.action_horizon, cfg.action_dim)
    _check(_np(v2), golden["mini16_v"], what="prefill + step")


def test_denoise_loop_kv_matches_golden(mini, golden):
    inp = mini.inputs()
    cfg = mini.cfg
    pm = O.prefix_mask(cfg.prefix_len)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    k, v = mini.rt.prefill(inp["prefix"], pm)
    x = mini.rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm)
    _check(_np(x), golden["mini16_loop"], what="loop")
    # replaying the captured graph with the same arguments gives the same bits
    x2 = mini.rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm)
    assert torch.equal(x, x2)


def test_loop_equals_host_stepped_loop_bitwise(mini):
    """compare_loop (python/mlc_vla/compare_loop.py): in-graph loop == host loop. Both paths run
    the same kernels on the same inputs, so the bits agree."""
    inp = mini.inputs(seed=5)
    cfg = mini.cfg
    pm = O.prefix_mask(cfg.prefix_len)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    n = cfg.num_denoise_steps
    te = O.time_embs(n, cfg.action_expert.width)
    k, v = mini.rt.prefill(inp["prefix"], pm)
    xg = _np(mini.rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm))
    x = inp["noise"].astype(np.float32)
    for i in range(n):
        vv = _np(mini.rt.denoise_step_kv(k, v, x.astype(np.float16), te[i:i + 1], sc, ss, pm))
        x = x + (-1.0 / n) * vv
    assert cosine(x, xg) >= 0.99999
    assert np.array_equal(x, xg)


def test_prefill_then_step_back_to_back_in_one_graph(mini):
    """prefill immediately followed by denoise_step_kv with nothing between them on the device
    (both captured into one CUDA graph, the step's first kernel launched programmatically after
    the prefill's last, which writes the last layer's K/V): the same bits as the two calls run
    apart. The caches are refilled with a sentinel before the replay, so a read that ran ahead
    of the prefill's writes would show."""
    cfg = mini.cfg
    rt = mini.rt
    dev = rt.device
    inp = mini.inputs(seed=7)
    pm = torch.from_numpy(O.prefix_mask(cfg.prefix_len)).to(dev)
    sc, ss = [torch.from_numpy(np.ascontiguousarray(a)).to(dev)
              for a in O.suffix_rope(cfg, cfg.prefix_len)]
    prefix = torch.from_numpy(inp["prefix"]).to(dev, torch.float16)
    x = torch.from_numpy(inp["x_t"]).to(dev, torch.float16)
    te = torch.from_numpy(inp["time_emb"]).reshape(1, -1).to(dev, torch.float16)
    vlm = cfg.vlm
    shape = (vlm.depth, 1, vlm.num_kv_heads, cfg.prefix_len, vlm.head_dim)
    k1 = torch.empty(shape, device=dev)
    v1 = torch.empty(shape, device=dev, dtype=torch.float16)
    o1 = torch.empty((1, cfg.action_horizon, cfg.action_dim), device=dev)
    rt.prefill(prefix, pm, keys=k1, values=v1)
    torch.cuda.synchronize()
    rt.denoise_step_kv(k1, v1, x, te, sc, ss, pm, out=o1)
    torch.cuda.synchronize()
    k2, v2, o2 = torch.empty_like(k1), torch.empty_like(v1), torch.empty_like(o1)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        rt.prefill(prefix, pm, keys=k2, values=v2)
        rt.denoise_step_kv(k2, v2, x, te, sc, ss, pm, out=o2)
    for _ in range(3):
        k2.fill_(1e4)
        v2.fill_(1e4)
        o2.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert rt.device_error() == 0
        assert torch.equal(k1, k2) and torch.equal(v1, v2) and torch.equal(o1, o2)
    del g


def test_batch_of_requests_matches_single(mini):
    """Independent requests in one call (own prefix, pad mask, RoPE offset) equal B=1 calls."""
    cfg = mini.cfg
    b = 3
    inp = mini.inputs(seed=2, batch=b)
    nvs = [cfg.prefix_len, cfg.prefix_len - 7, cfg.prefix_len // 2]
    pm = np.concatenate([O.prefix_mask(cfg.prefix_len, nv) for nv in nvs], 0)
    rope = [O.suffix_rope(cfg, nv) for nv in nvs]
    sc = np.concatenate([r[0] for r in rope], 0)
    ss = np.concatenate([r[1] for r in rope], 0)
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    k, v = mini.rt.prefill(inp["prefix"], pm)
    xb = _np(mini.rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm))
    for i in range(b):
        k1, v1 = mini.rt.prefill(inp["prefix"][i:i + 1], pm[i:i + 1])
        np.testing.assert_allclose(_np(k1)[:, 0], _np(k)[:, i], rtol=0, atol=1e-6 * 0 + 2e-3)
        x1 = _np(mini.rt.denoise_loop_kv(k1, v1, inp["noise"][i:i + 1], te, sc[i:i + 1],
                                         ss[i:i + 1], pm[i:i + 1]))
        _check(x1, xb[i:i + 1], 0.99999, 1e-2, f"batch row {i}")
        # and against the oracle with the same padding
        ko, vo = mini.oracle_kv(inp["prefix"][i:i + 1], pm[i:i + 1])
        xo = O.denoise_loop_kv(mini.p, cfg, ko, vo, inp["noise"][i:i + 1], te, sc[i:i + 1],
                               ss[i:i + 1], pm[i:i + 1])
        _check(x1, xo, what=f"padded request {i} vs oracle")


def test_pad_invariance():
    """compare_pad (python/mlc_vla/compare_pad.py:62-91) on the GPU: garbage pad tokens that
    the mask hides do not change v."""
    import dataclasses

    pad = 5
    full = config(recipes.MINI)
    trunc = dataclasses.replace(full, max_token_len=full.max_token_len - pad)
    mf, mt = Model(full), Model(trunc)
    P, V = full.prefix_len, trunc.prefix_len
    rng = np.random.default_rng(0)
    prefix = (0.02 * rng.standard_normal((1, P, full.vlm.width))).astype(np.float32)
    prefix[:, V:] = 10.0 * rng.standard_normal((1, pad, full.vlm.width))
    x_t = np.zeros((1, full.action_horizon, full.action_dim), np.float32)
    te = O.sinusoidal_time_emb(0.7, full.action_expert.width)

    def run(m, pre):
        pm = O.prefix_mask(m.cfg.prefix_len, num_valid=V)
        k, v = m.rt.prefill(pre, pm)
        sc, ss = O.suffix_rope(m.cfg, V)
        return _np(m.rt.denoise_step_kv(k, v, x_t, te, sc, ss, pm))

    a, b = run(mf, prefix), run(mt, prefix[:, :V].copy())
    assert cosine(a, b) >= 0.9999


@pytest.mark.parametrize("kw,dtype", [(recipes.DUMMY, "float16"), (recipes.MINI, "bfloat16")])
def test_other_shapes_and_dtypes_match_oracle(kw, dtype):
    m = Model(config(kw, dtype))
    cfg = m.cfg
    inp = m.inputs()
    pm = O.prefix_mask(cfg.prefix_len)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    k, v = m.rt.prefill(inp["prefix"], pm)
    x = _np(m.rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm))
    ko, vo = m.oracle_kv(inp["prefix"], pm)
    xo = O.denoise_loop_kv(m.p, cfg, ko, vo, inp["noise"], te, sc, ss, pm)
    tol = MAXABS if dtype == "float16" else 8e-2
    _check(x, xo, 0.999 if dtype == "bfloat16" else COS, tol, f"{kw['paligemma_variant']} {dtype}")


def test_full_width_two_layers_matches_oracle():
    """Every π0.5 width (2048 / 1024, MLP 16384 / 4096, 8 heads × 256, P=968, S=50, D=32) with
    two layers: prefill K/V, one step and the 10-step loop against the oracle."""
    m = Model(config(recipes.FULL2))
    cfg = m.cfg
    inp = m.inputs()
    nv = 868  # last 100 prefix positions padded
    pm = O.prefix_mask(cfg.prefix_len, nv)
    sc, ss = O.suffix_rope(cfg, nv)
    k, v = m.rt.prefill(inp["prefix"], pm)
    ko, vo = m.oracle_kv(inp["prefix"], pm)
    _check(_np(k), ko, 0.99999, 1e-2 * np.abs(ko).max(), "full-width keys")
    _check(_np(v), vo, 0.99999, 1e-2 * np.abs(vo).max(), "full-width values")
    vs = _np(m.rt.denoise_step_kv(k, v, inp["x_t"], inp["time_emb"], sc, ss, pm))
    vso = O.denoise_step_kv(m.p, cfg, ko, vo, inp["x_t"], inp["time_emb"], sc, ss, pm)
    _check(vs, vso, what="full-width step")
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    x = _np(m.rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm))
    xo = O.denoise_loop_kv(m.p, cfg, ko, vo, inp["noise"], te, sc, ss, pm)
    _check(x, xo, what="full-width loop")


def test_errors_are_raised_not_silent(mini):
    from mlc_vla._lib import Pi0Error

    cfg = mini.cfg
    with pytest.raises(ValueError):
        mini.rt.prefill(np.zeros((5, cfg.prefix_len, cfg.vlm.width), np.float32),
                        O.prefix_mask(cfg.prefix_len))  # batch 5 > max_batch 4
    from mlc_vla.runtime import Pi0Runtime

    rt = Pi0Runtime(cfg, device=0)
    with pytest.raises(Pi0Error, match="set_params"):
        rt.prefill(np.zeros((1, cfg.prefix_len, cfg.vlm.width), np.float32),
                   O.prefix_mask(cfg.prefix_len))


@pytest.mark.parametrize("preset", ["q4f16_1", "q4bf16_1", "q3f16_1"])
def test_gpu_quantiser_bit_exact(preset):
    from mlc_vla.quant import PRESETS
    from oracle import quant_oracle as Q

    q = PRESETS[preset]
    rng = np.random.default_rng(3)
    w = (0.02 * rng.standard_normal((96, 1000))).astype(np.float32)
    w[5, :40] = 0  # an all-zero group
    tdt = torch.float16 if q.model_dtype == "float16" else torch.bfloat16
    wt = torch.from_numpy(w).to("cuda", tdt)
    qw, qs = q.quantize_weight(wt)
    oq, os_ = Q.quantize(wt.float().cpu().numpy(), preset)
    assert np.array_equal(qw.cpu().numpy().view(np.uint32), oq)
    assert np.array_equal(qs.float().cpu().numpy(), os_)
    dq = q.dequantize(qw, qs, 1000)
    assert np.array_equal(dq.float().cpu().numpy(), Q.dequantize(oq, os_, preset, 1000))


def test_batch_beyond_weight_streaming_rows():
    """20 padded requests in one call: 20·S = 160 activation rows in the denoise step, more than
    the weight-streaming GEMM takes (128), so the tile GEMM with a separate norm runs instead.
    Every request (own prefix, pad mask and suffix RoPE offset) is checked against the oracle."""
    cfg = config(recipes.MINI)
    b = 20
    m = Model(cfg, max_batch=b)
    inp = m.inputs(seed=5, batch=b)
    rng = np.random.default_rng(9)
    nvs = [int(v) for v in rng.integers(cfg.prefix_len // 2, cfg.prefix_len + 1, size=b)]
    pm = np.concatenate([O.prefix_mask(cfg.prefix_len, nv) for nv in nvs], 0)
    rope = [O.suffix_rope(cfg, nv) for nv in nvs]
    sc = np.concatenate([r[0] for r in rope], 0)
    ss = np.concatenate([r[1] for r in rope], 0)
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    k, v = m.rt.prefill(inp["prefix"], pm)
    xb = _np(m.rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm))
    assert m.rt.device_error() == 0
    for i in (0, 7, 19):
        ko, vo = m.oracle_kv(inp["prefix"][i:i + 1], pm[i:i + 1])
        xo = O.denoise_loop_kv(m.p, cfg, ko, vo, inp["noise"][i:i + 1], te, sc[i:i + 1],
                               ss[i:i + 1], pm[i:i + 1])
        _check(xb[i:i + 1], xo, what=f"batch-20 request {i} (valid {nvs[i]})")


def test_m0_denoise_step_matches_oracle_and_m1(mini):
    """vm["denoise_step"] (M0 joint step, pi0_model.py:111-125) on the GPU: against the oracle's
    M0 step (gemma_dual.py:162-233 restated) and bit-identical to prefill + denoise_step_kv with
    an all-valid prefix (the M1 ≡ M0 identity, compare_kv.py:39-116)."""
    cfg = mini.cfg
    inp = mini.inputs(seed=4)
    v0 = _np(mini.rt.denoise_step(inp["prefix"], inp["x_t"], inp["time_emb"]))
    assert mini.rt.device_error() == 0
    vo = O.denoise_step(mini.p, cfg, inp["prefix"], inp["x_t"], inp["time_emb"])
    _check(v0, vo, what="M0 denoise_step vs oracle M0")
    pm = O.prefix_mask(cfg.prefix_len)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    k, v = mini.rt.prefill(inp["prefix"], pm)
    v1 = _np(mini.rt.denoise_step_kv(k, v, inp["x_t"], inp["time_emb"], sc, ss, pm))
    assert np.array_equal(v0, v1)
    # VM-style call, as the reference's compare_kv.py makes it
    v2 = mini.rt["denoise_step"](inp["prefix"], inp["x_t"], inp["time_emb"], mini.params)
    assert np.array_equal(v2.numpy(), v0)


def test_m0_equals_m1_full_width():
    """The M1 ≡ M0 gate at every π0.5 width (two layers): both computed on the GPU, bit-identical,
    and the M0 step within the fp16 tolerance of the oracle."""
    cfg = config(recipes.FULL2)
    m = Model(cfg)
    inp = m.inputs(seed=6)
    v0 = _np(m.rt.denoise_step(inp["prefix"], inp["x_t"], inp["time_emb"]))
    pm = O.prefix_mask(cfg.prefix_len)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    k, v = m.rt.prefill(inp["prefix"], pm)
    v1 = _np(m.rt.denoise_step_kv(k, v, inp["x_t"], inp["time_emb"], sc, ss, pm))
    assert m.rt.device_error() == 0
    assert np.array_equal(v0, v1)
    ko, vo = m.oracle_kv(inp["prefix"], pm)
    vref = O.denoise_step_kv(m.p, cfg, ko, vo, inp["x_t"], inp["time_emb"], sc, ss, pm)
    _check(v0, vref, what="M0 full width vs oracle")


@pytest.mark.parametrize("kw,dtype,logits", [
    (recipes.MINI, "float16", "float16"), (recipes.MINI, "bfloat16", "bfloat16"),
    (recipes.DUMMY, "float16", "float16"), (recipes.FULL2, "float16", "float16")])
def test_model_dtype_logits_match_oracle(kw, dtype, logits):
    """attn_logits_dtype set to the model dtype (the reference's tensor-core option,
    pi0_config.py:97-102, gemma_dual.py:115: q and k cast to fp16 / bf16 before q·kᵀ) against
    the oracle computing the same cast; the default "float32" is what every other test runs."""
    m = Model(config(kw, dtype, attn_logits_dtype=logits))
    cfg = m.cfg
    inp = m.inputs()
    pm = O.prefix_mask(cfg.prefix_len)
    sc, ss = O.suffix_rope(cfg, cfg.prefix_len)
    te = O.time_embs(cfg.num_denoise_steps, cfg.action_expert.width)
    k, v = m.rt.prefill(inp["prefix"], pm)
    ko, vo = m.oracle_kv(inp["prefix"], pm)
    _check(_np(k), ko, 0.99999, 1e-2 * np.abs(ko).max(), f"{logits} logits keys")
    x = _np(m.rt.denoise_loop_kv(k, v, inp["noise"], te, sc, ss, pm))
    xo = O.denoise_loop_kv(m.p, cfg, ko, vo, inp["noise"], te, sc, ss, pm)
    tol = MAXABS if dtype == "float16" else 8e-2
    _check(x, xo, 0.999 if dtype == "bfloat16" else COS, tol,
           f"{kw['paligemma_variant']} {dtype} {logits} logits")


def test_unsupported_logits_dtype_is_refused():
    from mlc_vla.runtime import Pi0Runtime

    with pytest.raises(ValueError, match="attn_logits_dtype"):
        Pi0Runtime(config(recipes.MINI, "float16", attn_logits_dtype="bfloat16"), device=0)

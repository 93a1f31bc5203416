"""CPU oracle for the π0.5 M1 hot path — TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and
its ``--impl reference`` arm) may import this module, and only as the checker or as the
timed CPU restatement of the reference; the product path (``mlc_vla`` + ``libpi0b200.so``)
never calls it.

This is a numpy restatement of the reference's M1 math, with the reference's dtype
placement made explicit: every tensor the reference keeps in the model dtype is rounded to
that dtype here (``rnd``), and everything the reference computes in fp32 stays fp32.

Followed code (paths relative to the reference project):

* ``python/mlc_vla/model/pi0/gemma_dual.py:24-57``   RoPE tables and half-split rotation
* ``gemma_dual.py:75-89``                            RMSNorm (plain and adaRMS)
* ``gemma_dual.py:91-94``                            gated residual
* ``gemma_dual.py:97-122``                           SDPA (fp32 logits, probs to model dtype)
* ``gemma_dual.py:132-135``                          GeGLU MLP
* ``gemma_dual.py:236-275,334-351,398-433``          prefill_e0 / decode_e1 / prefill_prefix /
                                                     decode_suffix
* ``gemma_dual.py:162-233,293-331,373-390``          M0 joint forward (for the M1≡M0 gate)
* ``python/mlc_vla/model/pi0/pi0_model.py:29-41``    joint additive mask
* ``pi0_model.py:106-194``                           _time_cond, denoise_step (M0), prefill,
                                                     denoise_step_kv, denoise_loop_kv
* ``pi0_model.py:101-104``                           embed_language (gather · sqrt(width))

Rounding conventions (the reference's TVM lowering is not available to pin them to the
ulp): a model-dtype matmul accumulates in fp32 and rounds once; a Linear with bias rounds
after the matmul and again after the bias add (``nn.Linear.forward`` is matmul then add);
GELU-tanh and SiLU are evaluated in fp32 and rounded once.

Pinning: the fp32 path is checked against the reference's own torch golden implementation
``python/mlc_vla/openpi_ref.py:92-214`` (``_SelfContainedRef``) by
``tests/golden/make_golden.py``, which commits the reference outputs as fixtures.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence

import numpy as np

Params = Dict[str, np.ndarray]

F32 = np.float32


# --------------------------------------------------------------------------------------------
# dtype emulation
# --------------------------------------------------------------------------------------------
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to bfloat16 (round to nearest even); returns fp32 holding them."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(F32)


def rnd(x, dtype: str) -> np.ndarray:
    """Round to the model dtype (fp32 storage of fp16/bf16 values)."""
    x = np.asarray(x, dtype=F32)
    if dtype == "float32":
        return x
    if dtype == "float16":
        return x.astype(np.float16).astype(F32)
    if dtype == "bfloat16":
        return bf16_round(x)
    raise ValueError(f"unsupported dtype {dtype}")


def prepare_params(params: Params, dtype: str) -> Params:
    """Model-dtype values of every parameter, held as fp32 (done once, outside timing)."""
    return {k: rnd(v, dtype) if v.dtype != np.uint32 else v for k, v in params.items()}


# --------------------------------------------------------------------------------------------
# elementwise pieces
# --------------------------------------------------------------------------------------------
def linear(x, w, b, dtype):
    """``nn.Linear``: matmul in the model dtype (fp32 accumulate, one rounding), then bias."""
    y = rnd(np.matmul(x, w.T), dtype)
    if b is not None:
        y = rnd(y + b, dtype)
    return y


def gelu_tanh(x):
    """GELU, tanh approximation: 0.5·x·(1 + tanh(√(2/π)·(x + 0.044715·x³)))."""
    x = x.astype(F32)
    c = F32(math.sqrt(2.0 / math.pi))
    return (F32(0.5) * x * (F32(1.0) + np.tanh(c * (x + F32(0.044715) * x * x * x)))).astype(F32)


def silu(x):
    x = x.astype(F32)
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def _normed(x, eps):
    """``gemma_dual.py:76-78``: x / sqrt(mean(x²) + eps) in fp32."""
    var = np.sum(x * x, axis=-1, keepdims=True, dtype=F32) / F32(x.shape[-1])
    return x / np.sqrt(var + F32(eps))


def rms_norm(x, w, eps, dtype):
    """Plain Gemma RMSNorm (``gemma_dual.py:79-82``): normed·(1+w), cast to the model dtype."""
    return rnd(_normed(x, eps) * (F32(1.0) + w), dtype)


def ada_rms_norm(x, mod, eps, dtype):
    """adaRMS (``gemma_dual.py:83-88``). ``mod`` [B,3W] is the model-dtype modulation.

    Returns (normed·(1+scale)+shift cast to the model dtype, gate in the model dtype).
    """
    w = x.shape[-1]
    mod = mod.reshape(mod.shape[0], 1, 3 * w)
    scale, shift, gate = mod[..., :w], mod[..., w:2 * w], mod[..., 2 * w:]
    out = _normed(x, eps) * (F32(1.0) + scale) + shift
    return rnd(out, dtype), gate


def gated_residual(x, y, gate, dtype):
    """``gemma_dual.py:91-94``: x + y (prefix) or x + y·gate (suffix), model dtype."""
    if gate is None:
        return rnd(x + y, dtype)
    return rnd(x + rnd(y * gate, dtype), dtype)


def rope_tables(num_positions: int, head_dim: int, theta: float, offset: int = 0):
    """``gemma_dual.py:24-44`` / ``sample.py:38-47``: cos/sin [L, hd/2] fp32 from float64."""
    half = head_dim // 2
    pos = np.arange(offset, offset + num_positions, dtype=np.float64)
    freq_exp = (2.0 / head_dim) * np.arange(half, dtype=np.float64)
    timescale = theta ** freq_exp
    rad = pos[:, None] / timescale[None, :]
    return np.cos(rad).astype(F32), np.sin(rad).astype(F32)


def apply_rope(x, cos, sin):
    """``gemma_dual.py:47-57``: x [B,T,n,hd] (model dtype) → fp32 rotated; cos/sin [B|1,T,hd/2]."""
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    c = cos[:, :, None, :]
    s = sin[:, :, None, :]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1).astype(F32)


def sdpa(q, k, v, mask, dtype, logits_dtype="float32"):
    """``gemma_dual.py:97-122``.

    q [B,n,Tq,hd] fp32 (rotated, scaled); k [B,kv,Ts,hd] fp32; v [B,kv,Ts,hd] model dtype;
    mask additive fp32 broadcastable to [B,n,Tq,Ts]. Returns [B,Tq,n*hd] in the model dtype.
    """
    b, n, tq, hd = q.shape
    kv = k.shape[1]
    if kv != n:
        k = np.repeat(k, n // kv, axis=1)
        v = np.repeat(v, n // kv, axis=1)
    if logits_dtype != "float32":
        q, k = rnd(q, logits_dtype), rnd(k, logits_dtype)
    logits = np.matmul(q, np.swapaxes(k, -1, -2)).astype(F32)
    if mask is not None:
        logits = logits + mask.astype(F32)
    m = np.max(logits, axis=-1, keepdims=True)
    e = np.exp(logits - m)
    probs = rnd(e / np.sum(e, axis=-1, keepdims=True, dtype=F32), dtype)
    enc = rnd(np.matmul(probs, v), dtype)
    return np.ascontiguousarray(np.swapaxes(enc, 1, 2)).reshape(b, tq, n * hd)


def mlp(x, w_gu, w_d, dtype):
    """``gemma_dual.py:132-135``: down(gelu_tanh(gate)·up) with gate rows before up rows."""
    gu = linear(x, w_gu, None, dtype)
    f = w_gu.shape[0] // 2
    h = rnd(rnd(gelu_tanh(gu[..., :f]), dtype) * gu[..., f:], dtype)
    return linear(h, w_d, None, dtype)


# --------------------------------------------------------------------------------------------
# model pieces
# --------------------------------------------------------------------------------------------
class Dims:
    """Sizes read from a Pi0Config-like object (duck-typed: .vlm, .action_expert, ...)."""

    def __init__(self, cfg):
        self.cfg = cfg
        self.L = cfg.vlm.depth
        self.H = cfg.vlm.num_heads
        self.KV = cfg.vlm.num_kv_heads
        self.hd = cfg.vlm.head_dim
        self.W0 = cfg.vlm.width
        self.W1 = cfg.action_expert.width
        self.P = cfg.prefix_len
        self.S = cfg.suffix_len
        self.D = cfg.action_dim
        self.dt = cfg.dtype
        self.eps = cfg.rms_norm_eps
        self.theta = cfg.rope_theta
        self.logits_dtype = getattr(cfg, "attn_logits_dtype", "float32")


def _lay(i):
    return f"backbone.layers.{i}."


def time_cond(p: Params, time_emb, dt):
    """``pi0_model.py:106-109``: silu(time_mlp_out(silu(time_mlp_in(te))))."""
    x = rnd(silu(linear(time_emb, p["time_mlp_in.weight"], p["time_mlp_in.bias"], dt)), dt)
    return rnd(silu(linear(x, p["time_mlp_out.weight"], p["time_mlp_out.bias"], dt)), dt)


def modulation(p: Params, prefix: str, cond, dt):
    return linear(cond, p[prefix + ".modulation.weight"], p[prefix + ".modulation.bias"], dt)


def prefill(p: Params, cfg, prefix_embs, prefix_mask):
    """``pi0_model.py:128-140`` → ``gemma_dual.py:398-415``.

    prefix_embs [B,P,W0] (any float dtype), prefix_mask [B|1,1,1,P] fp32.
    Returns keys [L,B,KV,P,hd] fp32 and values [L,B,KV,P,hd] (model-dtype values in fp32).
    """
    d = Dims(cfg)
    dt = d.dt
    x = rnd(prefix_embs, dt)
    b = x.shape[0]
    cos, sin = rope_tables(d.P, d.hd, d.theta, 0)
    cos, sin = cos[None], sin[None]
    keys = np.zeros((d.L, b, d.KV, d.P, d.hd), F32)
    values = np.zeros((d.L, b, d.KV, d.P, d.hd), F32)
    for i in range(d.L):
        pre = _lay(i)
        a = pre + "self_attn.experts.0."
        n = rms_norm(x, p[pre + "input_layernorm.0.weight"], d.eps, dt)
        k = linear(n, p[a + "k_proj.weight"], None, dt).reshape(b, d.P, d.KV, d.hd)
        v = linear(n, p[a + "v_proj.weight"], None, dt).reshape(b, d.P, d.KV, d.hd)
        kr = apply_rope(k, cos, sin)
        keys[i] = np.swapaxes(kr, 1, 2)
        values[i] = np.swapaxes(v, 1, 2)
        if i == d.L - 1:
            break  # the prefix hidden state after the last layer is never read
        q = linear(n, p[a + "q_proj.weight"], None, dt).reshape(b, d.P, d.H, d.hd)
        q = apply_rope(q, cos, sin) * F32(d.hd ** -0.5)
        enc = sdpa(np.swapaxes(q, 1, 2), keys[i], values[i], prefix_mask, dt, d.logits_dtype)
        x = gated_residual(x, linear(enc, p[a + "o_proj.weight"], None, dt), None, dt)
        n2 = rms_norm(x, p[pre + "post_attention_layernorm.0.weight"], d.eps, dt)
        x = gated_residual(x, mlp(n2, p[pre + "mlp.0.gate_up_proj.weight"],
                                  p[pre + "mlp.0.down_proj.weight"], dt), None, dt)
    return keys, values


def suffix_mods(p: Params, cfg, cond):
    """The 2·L+1 adaRMS modulations of one step (they depend on the time condition only)."""
    d = Dims(cfg)
    mods = []
    for i in range(d.L):
        for ln in ("input_layernorm", "post_attention_layernorm"):
            mods.append(modulation(p, f"{_lay(i)}{ln}.1", cond, d.dt))
    mods.append(modulation(p, "backbone.final_norm.1", cond, d.dt))
    return mods


def decode_suffix(p: Params, cfg, emb, keys, values, cond, scos, ssin, full_mask):
    """``gemma_dual.py:417-433`` with ``decode_e1`` (``:343-351``) and ``attn_decode_e1``
    (``:255-275``). emb [B,S,W1] model dtype; scos/ssin [B|1,S,hd/2]; full_mask
    [B|1,1,1,P+S]. Returns the final-norm suffix hidden state [B,S,W1]."""
    d = Dims(cfg)
    dt = d.dt
    x = emb
    b = x.shape[0]
    mods = suffix_mods(p, cfg, cond)
    for i in range(d.L):
        pre = _lay(i)
        a = pre + "self_attn.experts.1."
        n, gate = ada_rms_norm(x, mods[2 * i], d.eps, dt)
        q = linear(n, p[a + "q_proj.weight"], None, dt).reshape(b, d.S, d.H, d.hd)
        k = linear(n, p[a + "k_proj.weight"], None, dt).reshape(b, d.S, d.KV, d.hd)
        v = linear(n, p[a + "v_proj.weight"], None, dt).reshape(b, d.S, d.KV, d.hd)
        q = apply_rope(q, scos, ssin) * F32(d.hd ** -0.5)
        k = apply_rope(k, scos, ssin)
        kfull = np.concatenate([keys[i], np.swapaxes(k, 1, 2)], axis=2)
        vfull = np.concatenate([values[i], np.swapaxes(v, 1, 2)], axis=2)
        enc = sdpa(np.swapaxes(q, 1, 2), kfull, vfull, full_mask, dt, d.logits_dtype)
        x = gated_residual(x, linear(enc, p[a + "o_proj.weight"], None, dt), gate, dt)
        n2, gate2 = ada_rms_norm(x, mods[2 * i + 1], d.eps, dt)
        x = gated_residual(x, mlp(n2, p[pre + "mlp.1.gate_up_proj.weight"],
                                  p[pre + "mlp.1.down_proj.weight"], dt), gate2, dt)
    out, _ = ada_rms_norm(x, mods[-1], d.eps, dt)
    return out


def _full_mask(prefix_mask, s):
    pm = np.asarray(prefix_mask, F32)
    z = np.zeros(pm.shape[:-1] + (s,), F32)
    return np.concatenate([pm, z], axis=-1)


def _rope_arg(t):
    t = np.asarray(t, F32)
    return t.reshape(t.shape[0], t.shape[1], t.shape[-1])  # [B,S,1,hd/2] → [B,S,hd/2]


def denoise_step_kv(p: Params, cfg, keys, values, x_t, time_emb, suffix_cos, suffix_sin,
                    prefix_mask):
    """``pi0_model.py:142-163``. Returns v [B,S,D] fp32."""
    d = Dims(cfg)
    dt = d.dt
    emb = linear(rnd(x_t, dt), p["action_in_proj.weight"], p["action_in_proj.bias"], dt)
    cond = time_cond(p, rnd(time_emb, dt), dt)
    out = decode_suffix(p, cfg, emb, keys, values, cond, _rope_arg(suffix_cos),
                        _rope_arg(suffix_sin), _full_mask(prefix_mask, d.S))
    return linear(out, p["action_out_proj.weight"], p["action_out_proj.bias"], dt).astype(F32)


def denoise_loop_kv(p: Params, cfg, keys, values, x0, time_embs, suffix_cos, suffix_sin,
                    prefix_mask, num_steps: Optional[int] = None):
    """``pi0_model.py:165-194``: N unrolled Euler steps, x fp32, dt = -1/N (fp32)."""
    d = Dims(cfg)
    dt = d.dt
    n = cfg.num_denoise_steps if num_steps is None else num_steps
    step = F32(-1.0 / n)
    fm = _full_mask(prefix_mask, d.S)
    sc, ss = _rope_arg(suffix_cos), _rope_arg(suffix_sin)
    te = rnd(time_embs, dt)
    x = np.asarray(x0, F32)
    for i in range(n):
        emb = linear(rnd(x, dt), p["action_in_proj.weight"], p["action_in_proj.bias"], dt)
        cond = time_cond(p, te[i:i + 1], dt)
        out = decode_suffix(p, cfg, emb, keys, values, cond, sc, ss, fm)
        v = linear(out, p["action_out_proj.weight"], p["action_out_proj.bias"], dt).astype(F32)
        x = (x + step * v).astype(F32)
    return x


def joint_additive_mask(prefix_len, suffix_len, neg_inf, dtype):
    """``pi0_model.py:29-41``: prefix sees prefix; suffix sees prefix and all of suffix."""
    total = prefix_len + suffix_len
    att = np.zeros(total, np.int32)
    att[prefix_len] = 1
    cs = np.cumsum(att)
    allow = cs[None, :] <= cs[:, None]
    m = np.where(allow, 0.0, neg_inf).astype(F32)
    if dtype == "float16":
        with np.errstate(over="ignore"):
            m = m.astype(np.float16).astype(F32)  # -2.38e38 saturates to -inf in fp16
    elif dtype == "bfloat16":
        m = bf16_round(m)
    return m.reshape(1, 1, total, total)


def denoise_step(p: Params, cfg, prefix_embs, x_t, time_emb):
    """M0 joint step (``pi0_model.py:111-125`` → ``gemma_dual.py:162-233,293-331,373-390``)."""
    d = Dims(cfg)
    dt = d.dt
    total = d.P + d.S
    cos, sin = rope_tables(total, d.hd, d.theta, 0)
    cos, sin = cos[None], sin[None]
    mask = joint_additive_mask(d.P, d.S, cfg.attn_neg_inf, dt)
    suffix = linear(rnd(x_t, dt), p["action_in_proj.weight"], p["action_in_proj.bias"], dt)
    cond = time_cond(p, rnd(time_emb, dt), dt)
    xs = [rnd(prefix_embs, dt), suffix]
    b = xs[0].shape[0]
    for i in range(d.L):
        pre = _lay(i)
        normed, gates = [], []
        for e in range(2):
            if e == 0:
                normed.append(rms_norm(xs[0], p[pre + "input_layernorm.0.weight"], d.eps, dt))
                gates.append(None)
            else:
                nn_, g = ada_rms_norm(xs[1], modulation(p, pre + "input_layernorm.1", cond, dt),
                                      d.eps, dt)
                normed.append(nn_)
                gates.append(g)
        qs, ks, vs = [], [], []
        for e in range(2):
            a = f"{pre}self_attn.experts.{e}."
            t = normed[e].shape[1]
            qs.append(linear(normed[e], p[a + "q_proj.weight"], None, dt).reshape(b, t, d.H, d.hd))
            ks.append(linear(normed[e], p[a + "k_proj.weight"], None, dt).reshape(b, t, d.KV, d.hd))
            vs.append(linear(normed[e], p[a + "v_proj.weight"], None, dt).reshape(b, t, d.KV, d.hd))
        q = apply_rope(np.concatenate(qs, 1), cos, sin) * F32(d.hd ** -0.5)
        k = apply_rope(np.concatenate(ks, 1), cos, sin)
        v = np.concatenate(vs, 1)
        enc = sdpa(np.swapaxes(q, 1, 2), np.swapaxes(k, 1, 2), np.swapaxes(v, 1, 2), mask, dt,
                   d.logits_dtype)
        chunks = [enc[:, :d.P], enc[:, d.P:]]
        new = []
        for e in range(2):
            a = f"{pre}self_attn.experts.{e}."
            x1 = gated_residual(xs[e], linear(chunks[e], p[a + "o_proj.weight"], None, dt),
                                gates[e], dt)
            if e == 0:
                n2, g2 = rms_norm(x1, p[pre + "post_attention_layernorm.0.weight"], d.eps, dt), None
            else:
                n2, g2 = ada_rms_norm(x1, modulation(p, pre + "post_attention_layernorm.1", cond, dt),
                                      d.eps, dt)
            y = mlp(n2, p[f"{pre}mlp.{e}.gate_up_proj.weight"], p[f"{pre}mlp.{e}.down_proj.weight"], dt)
            new.append(gated_residual(x1, y, g2, dt))
        xs = new
    out, _ = ada_rms_norm(xs[1], modulation(p, "backbone.final_norm.1", cond, dt), d.eps, dt)
    return linear(out, p["action_out_proj.weight"], p["action_out_proj.bias"], dt).astype(F32)


# --------------------------------------------------------------------------------------------
# host tables (restated from python/mlc_vla/sample.py:27-74, openpi_ref.py:49-58)
# --------------------------------------------------------------------------------------------
def sinusoidal_time_emb(t: float, dim: int) -> np.ndarray:
    frac = np.linspace(0.0, 1.0, dim // 2, dtype=np.float64)
    period = 4e-3 * (4.0 / 4e-3) ** frac
    arg = (1.0 / period * 2 * math.pi)[None, :] * np.array([t], np.float64)[:, None]
    return np.concatenate([np.sin(arg), np.cos(arg)], axis=1).astype(F32)


def time_embs(n: int, dim: int) -> np.ndarray:
    t, dt = 1.0, -1.0 / n
    out = []
    for _ in range(n):
        out.append(sinusoidal_time_emb(t, dim))
        t += dt
    return np.concatenate(out, 0)


def prefix_mask(prefix_len: int, num_valid: Optional[int] = None, neg: float = -1e9):
    valid = np.ones(prefix_len, F32)
    if num_valid is not None:
        valid[:] = 0
        valid[:num_valid] = 1
    return np.where(valid > 0, 0.0, neg).astype(F32).reshape(1, 1, 1, prefix_len)


def suffix_rope(cfg, offset: int):
    c, s = rope_tables(cfg.suffix_len, cfg.vlm.head_dim, cfg.rope_theta, offset)
    return c.reshape(1, cfg.suffix_len, 1, -1), s.reshape(1, cfg.suffix_len, 1, -1)


def host_loop(p: Params, cfg, keys, values, noise, suffix_cos, suffix_sin, pmask, num_steps):
    """``sample.py:139-163`` + ``euler_loop`` (``:67-74``): per-step denoise_step_kv."""
    te = time_embs(num_steps, cfg.action_expert.width)
    x = np.asarray(noise, F32)
    step = -1.0 / num_steps
    for i in range(num_steps):
        v = denoise_step_kv(p, cfg, keys, values, rnd(x, cfg.dtype), te[i:i + 1], suffix_cos,
                            suffix_sin, pmask)
        x = (x + F32(step) * v).astype(F32)
    return x


# --------------------------------------------------------------------------------------------
# helpers for tests
# --------------------------------------------------------------------------------------------
def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-12))


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def random_params(named_params: Sequence, seed: int = 0, scale: float = 0.02) -> Params:
    """N(0, scale²) weights in parameter-table order (the reference tests' ``make_params``,
    ``python/tests/conftest.py:47-63``); integer parameters are zeros."""
    rng = np.random.default_rng(seed)
    out: Params = {}
    for name, spec in named_params:
        shape = tuple(int(s) for s in spec.shape)
        if str(spec.dtype).startswith(("int", "uint")):
            out[name] = np.zeros(shape, spec.dtype)
        else:
            out[name] = (scale * rng.standard_normal(shape)).astype(F32)
    return out


def embed_language(table, input_ids, dtype: str) -> np.ndarray:
    """pi0_model.py:101-104: ``embed_tokens(input_ids) * math.sqrt(width)`` with the table in the
    model dtype. The Python constant takes the tensor's dtype, so it is rounded to that dtype
    first; the product (exact in fp32) is rounded once. Ids outside the table give zero rows."""
    table = np.asarray(table)
    ids = np.asarray(input_ids).reshape(-1).astype(np.int64)
    width = table.shape[1]
    c = rnd(np.float32(math.sqrt(width)), dtype).astype(np.float32)
    ok = (ids >= 0) & (ids < table.shape[0])
    rows = rnd(table, dtype).astype(np.float32)[np.where(ok, ids, 0)]
    rows[~ok] = 0.0
    return rnd(rows * c, dtype)

"""M1 host driver: one prefill, then N suffix-only Euler steps (flow matching, t: 1 → 0).

Drop-in for the reference's ``python/mlc_vla/sample.py``: same helper functions and the same
``PiZeroRunner`` API (``__init__``, ``to_params``, ``sample``, ``sample_graph``), with the
TVM executable replaced by ``libpi0b200`` (``mlc_vla.runtime.Pi0Runtime``).

Helpers (bit-identical to the reference's, checked against its outputs in tests/golden):
  make_time_embs (sample.py:27-35), make_rope_np (:38-47), make_prefix_mask_np (:50-64),
  euler_loop (:67-74).

``PiZeroRunner`` extends the reference in one way: ``prefix_embs`` may carry a leading batch
of B ≤ ``max_batch`` independent requests (``prefix_pad`` then is [P] or [B, P]); with B = 1
every call behaves as the reference's.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from mlc_vla.compile import compile_model
from mlc_vla.model.pi0 import Pi0Config
from mlc_vla.openpi_ref import sinusoidal_time_emb
from mlc_vla.runtime import DeviceArray, to_device

_KV_FUNCS = ["prefill", "denoise_step_kv", "denoise_loop_kv"]


def make_time_embs(num_steps: int, ae_width: int) -> list:
    """Sinusoidal time embeddings for t = 1, 1 + dt, ... (dt = -1/N): N arrays [1, W1] fp32."""
    dt = -1.0 / num_steps
    t = 1.0
    embs = []
    for _ in range(num_steps):
        embs.append(sinusoidal_time_emb(t, ae_width))
        t += dt
    return embs


def make_rope_np(num_positions: int, head_dim: int, theta: float, offset: int = 0):
    """RoPE tables [1, L, 1, hd/2] fp32, computed in float64 (gemma_dual.py:24-44)."""
    half = head_dim // 2
    pos = np.arange(offset, offset + num_positions, dtype=np.float64)
    freq_exp = (2.0 / head_dim) * np.arange(half, dtype=np.float64)
    radians = pos[:, None] / (theta ** freq_exp)[None, :]
    cos = np.cos(radians).reshape(1, num_positions, 1, half).astype("float32")
    sin = np.sin(radians).reshape(1, num_positions, 1, half).astype("float32")
    return cos, sin


def make_prefix_mask_np(prefix_len: int, num_valid: Optional[int] = None,
                        pad_mask: Optional[np.ndarray] = None, neg: float = -1e9) -> np.ndarray:
    """Additive prefix mask [1, 1, 1, P]: 0 for valid tokens, `neg` for padding.

    `pad_mask` ([P] bool / 0-1) wins over `num_valid` (first num_valid tokens valid);
    neither means all valid."""
    valid = np.ones((prefix_len,), dtype=np.float32)
    if pad_mask is not None:
        valid = np.asarray(pad_mask, dtype=np.float32).reshape(-1)[:prefix_len]
    elif num_valid is not None:
        valid = np.zeros((prefix_len,), dtype=np.float32)
        valid[: int(num_valid)] = 1.0
    return np.where(valid > 0, 0.0, neg).astype("float32").reshape(1, 1, 1, prefix_len)


def euler_loop(step_fn, x0: np.ndarray, num_steps: int) -> np.ndarray:
    """x ← x + dt·v(x, i) for i < N with dt = -1/N, in fp32."""
    dt = -1.0 / num_steps
    x = x0.astype(np.float32)
    for i in range(num_steps):
        v = step_fn(x, i).astype(np.float32)
        x = x + dt * v
    return x


class PiZeroRunner:
    """Builds the M1 runtime on a B200 and drives the denoising loop from the host."""

    def __init__(self, config: Pi0Config, target: str = "cuda", cuda_graph: bool = False,
                 cublas=None, max_batch: int = 1, device: Optional[int] = None, quant=None):
        self.config = config
        self.target = target
        self.cuda_graph = cuda_graph
        self.ex, self.named_params = compile_model(config, target, functions=_KV_FUNCS,
                                                   cuda_graph=cuda_graph, cublas=cublas,
                                                   max_batch=max_batch, device=device,
                                                   quant=quant)
        # this build issues no cuBLAS call: every GEMM is one of its own kernels
        self.cublas = False
        self.dev = self.ex.device
        self.vm = self.ex
        self._stage = {}
        # device copies of tables derived from the inputs alone (pad mask + suffix RoPE per pad
        # pattern, time embeddings per step count): computed and uploaded once, not per call
        self._tables = {}

    def to_params(self, arrays):
        """Move numpy weights (ordered as ``named_params``) to the GPU."""
        return self.ex.to_params(arrays)

    # -- helpers --
    def _dt(self):
        return self.ex.dtype

    def _batch(self, prefix_embs) -> int:
        a = np.asarray(prefix_embs) if not isinstance(prefix_embs, torch.Tensor) else prefix_embs
        return int(a.shape[0]) if a.ndim == 3 else 1

    def _prepare(self, params, prefix_embs, prefix_pad):
        """Prefill the K/V cache and build the prefix pad mask and suffix RoPE tables.

        Returns (keys, values, prefix_mask, suffix_cos, suffix_sin, num_valid)."""
        cfg = self.config
        b = self._batch(prefix_embs)
        if prefix_pad is None:
            pads = [None] * b
        else:
            pp = np.asarray(prefix_pad).reshape(-1, cfg.prefix_len)
            pads = [pp[min(i, pp.shape[0] - 1)] for i in range(b)]
        prefix_mask, suffix_cos, suffix_sin, nvs = self._pad_tables(pads)
        dev = self.dev
        x = prefix_embs if isinstance(prefix_embs, torch.Tensor) else np.asarray(prefix_embs)
        # a pinned host prefix goes up without the host waiting for the copy (every caller of
        # _prepare reads its result back before returning, so the host buffer is free by then)
        prefix_dev = to_device(x, self._dt(), dev, non_blocking=True)
        st = self._staging(b)
        k, v = self.ex.prefill(prefix_dev, prefix_mask, params, keys=st["keys"], values=st["values"])
        keys, values = DeviceArray(k), DeviceArray(v)
        num_valid = nvs[0] if b == 1 else nvs
        return keys, values, prefix_mask, suffix_cos, suffix_sin, num_valid

    def _pad_tables(self, pads):
        """(prefix mask, suffix cos, suffix sin) on the device and the valid counts for one
        pad pattern per request (None = all valid), cached by the patterns' contents."""
        key = ("pad",) + tuple(None if p is None else np.asarray(p, np.float32).tobytes()
                               for p in pads)
        hit = self._tables.get(key)
        if hit is not None:
            return hit
        cfg = self.config
        hd = cfg.vlm.head_dim
        masks, coss, sins, nvs = [], [], [], []
        for pad in pads:
            if pad is None:
                nv = cfg.prefix_len
                m = make_prefix_mask_np(cfg.prefix_len)
            else:
                nv = int(np.asarray(pad).reshape(-1).sum())
                m = make_prefix_mask_np(cfg.prefix_len, pad_mask=pad)
            c, s = make_rope_np(cfg.suffix_len, hd, cfg.rope_theta, offset=nv)
            masks.append(m)
            coss.append(c)
            sins.append(s)
            nvs.append(nv)
        dev = self.dev
        out = (to_device(np.concatenate(masks, 0), "float32", dev),
               to_device(np.concatenate(coss, 0), "float32", dev),
               to_device(np.concatenate(sins, 0), "float32", dev), nvs)
        if len(self._tables) > 256:
            self._tables.clear()
        self._tables[key] = out
        return out

    def _time_table(self, n: int) -> torch.Tensor:
        """make_time_embs(n, W1) stacked [n, W1] in the model dtype, on the device (cached)."""
        key = ("time", n)
        if key not in self._tables:
            te = np.concatenate(make_time_embs(n, self.config.action_expert.width), axis=0)
            self._tables[key] = to_device(te, self._dt(), self.dev)
        return self._tables[key]

    def _noise(self, noise, seed, batch=1):
        cfg = self.config
        if noise is None:
            rng = np.random.default_rng(seed)
            noise = rng.standard_normal((batch, cfg.action_horizon, cfg.action_dim)).astype(np.float32)
        return np.asarray(noise).astype(np.float32)

    def sample(self, params, prefix_embs, noise=None, num_steps: int = 10, seed: int = 0,
               prefix_pad=None) -> np.ndarray:
        """Host Euler loop: one ``denoise_step_kv`` call per step with a host↔device round trip
        (x up, v down), exactly as the reference's ``sample`` (sample.py:139-163)."""
        cfg = self.config
        dt = self._dt()
        keys, values, pmask, scos, ssin, _ = self._prepare(params, prefix_embs, prefix_pad)
        b = self._batch(prefix_embs)
        noise = self._noise(noise, seed, b)
        time_embs = make_time_embs(num_steps, cfg.action_expert.width)
        te_dev = [to_device(te, dt, self.dev) for te in time_embs]

        def step_fn(x_np, i):
            x_dev = to_device(x_np, dt, self.dev)
            v = self.vm["denoise_step_kv"](keys, values, x_dev, te_dev[i], scos, ssin, pmask,
                                           params)
            return v.numpy()

        return euler_loop(step_fn, noise, num_steps)

    def sample_graph(self, params, prefix_embs, noise=None, seed: int = 0,
                     prefix_pad=None) -> np.ndarray:
        """In-graph loop: one ``denoise_loop_kv`` call (a replayed CUDA graph) runs all
        ``config.num_denoise_steps`` steps (sample.py:165-187)."""
        cfg = self.config
        n = cfg.num_denoise_steps
        keys, values, pmask, scos, ssin, _ = self._prepare(params, prefix_embs, prefix_pad)
        b = self._batch(prefix_embs)
        noise = self._noise(noise, seed, b)
        st = self._staging(b)
        # the noise goes up from a pinned staging buffer without a host wait (a pageable copy
        # would hold the host until the prefill has run, leaving the GPU idle while the loop is
        # launched); the previous call's copies finished before it returned
        st["x0_host"].copy_(torch.from_numpy(noise.reshape(st["x0"].shape)))
        st["x0"].copy_(st["x0_host"], non_blocking=True)
        # the loop's graph reads fixed buffers: refresh them only when the cached tables change
        src = (pmask.torch if isinstance(pmask, DeviceArray) else pmask, scos, ssin,
               self._time_table(n))
        if st.get("src") is None or any(old is not new for old, new in zip(st["src"], src)):
            for name, t in zip(("pmask", "scos", "ssin", "te"), src):
                st[name].copy_(t)
            st["src"] = src
        self.ex.denoise_loop_kv(keys.torch, values.torch, st["x0"], st["te"], st["scos"],
                                st["ssin"], st["pmask"], params, out=st["x"])
        return st["x"].cpu().numpy()

    def _staging(self, b):
        """Persistent device buffers for sample_graph, so the loop's CUDA graph is reused."""
        if b not in self._stage:
            cfg = self.config
            dev = self.dev
            half = cfg.vlm.head_dim // 2
            tdt = torch.float16 if self._dt() == "float16" else torch.bfloat16
            vlm = cfg.vlm
            kv = (vlm.depth, b, vlm.num_kv_heads, cfg.prefix_len, vlm.head_dim)
            self._stage[b] = {
                "keys": torch.empty(kv, dtype=torch.float32, device=dev),
                "values": torch.empty(kv, dtype=tdt, device=dev),
                "x0": torch.empty((b, cfg.action_horizon, cfg.action_dim), dtype=torch.float32, device=dev),
                "x0_host": torch.empty((b, cfg.action_horizon, cfg.action_dim), dtype=torch.float32,
                                       pin_memory=True),
                "x": torch.empty((b, cfg.action_horizon, cfg.action_dim), dtype=torch.float32, device=dev),
                "te": torch.empty((cfg.num_denoise_steps, cfg.action_expert.width), dtype=tdt, device=dev),
                "pmask": torch.empty((b, 1, 1, cfg.prefix_len), dtype=torch.float32, device=dev),
                "scos": torch.empty((b, cfg.suffix_len, 1, half), dtype=torch.float32, device=dev),
                "ssin": torch.empty((b, cfg.suffix_len, 1, half), dtype=torch.float32, device=dev),
            }
        return self._stage[b]

"""Python host for libpi0b200: one ``Pi0Runtime`` per (model, GPU).

``Pi0Runtime`` plays the role of the reference's compiled executable + ``relax.VirtualMachine``
(``python/mlc_vla/compile.py:99-133``, ``sample.py:91-95``): indexing it with an exported
function name gives a callable with the reference's argument order, packed params last
(``pi0_model.py:227-251``):

    keys, values = rt["prefill"](prefix_embs, prefix_mask, params)
    v            = rt["denoise_step_kv"](keys, values, x_t, time_emb, suffix_cos, suffix_sin,
                                         prefix_mask, params)
    x            = rt["denoise_loop_kv"](keys, values, x0, time_embs, suffix_cos, suffix_sin,
                                         prefix_mask, params)

Multi-output returns are tuples (``ret[0]``, ``ret[1]``); every returned tensor has
``.numpy()`` like a TVM NDArray. PyTorch provides device memory and the CUDA stream; all compute
happens in the library's kernels, on torch's current stream.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _lib
from .model.pi0.pi0_config import Pi0Config
from .model.pi0.pi0_model import ParamSpec, backbone_named_params

TORCH_DTYPE = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
               "uint32": torch.int32}


class DeviceArray:
    """A device tensor with the NDArray surface the reference's callers use (``.numpy()``,
    ``.shape``, ``.dtype``); ``.torch`` is the underlying tensor."""

    __slots__ = ("torch",)

    def __init__(self, t: torch.Tensor):
        self.torch = t

    @property
    def shape(self):
        return tuple(self.torch.shape)

    @property
    def dtype(self) -> str:
        return str(self.torch.dtype).replace("torch.", "")

    def numpy(self) -> np.ndarray:
        t = self.torch.detach()
        if t.dtype == torch.bfloat16:
            t = t.float()
        return t.cpu().numpy()

    def data_ptr(self) -> int:
        return self.torch.data_ptr()

    def __dlpack__(self, *a, **k):
        return self.torch.__dlpack__(*a, **k)

    def __dlpack_device__(self):
        return self.torch.__dlpack_device__()

    def __repr__(self):
        return f"DeviceArray(shape={self.shape}, dtype={self.dtype}, device={self.torch.device})"


def to_device(x, dtype: str, device, non_blocking: bool = False) -> torch.Tensor:
    """numpy / torch / DeviceArray -> contiguous torch tensor of `dtype` on `device`.

    `non_blocking`: a pinned host tensor is copied on the current stream without waiting for the
    copy; the caller must not reuse the host memory until it synchronises with that stream."""
    if isinstance(x, DeviceArray):
        x = x.torch
    if isinstance(x, torch.Tensor):
        t = x
    else:
        a = np.asarray(x)
        if a.dtype == np.float16 and dtype != "float16":
            a = a.astype(np.float32)
        if a.dtype == np.uint32:  # packed quantisation codes: keep the bits (int32 storage)
            a = a.view(np.int32)
        t = torch.from_numpy(np.ascontiguousarray(a))
    nb = non_blocking and t.device.type == "cpu" and t.is_pinned()
    return t.to(device=device, dtype=TORCH_DTYPE[dtype], non_blocking=nb).contiguous()


def config_struct(cfg: Pi0Config, max_batch: int = 1, quant=None) -> _lib.Pi0ConfigC:
    vlm, ae = cfg.vlm, cfg.action_expert
    dtype = quant.model_dtype if quant is not None else cfg.dtype
    if dtype not in ("float16", "bfloat16"):
        raise ValueError(
            f"the B200 build computes in float16 or bfloat16; config.dtype={cfg.dtype!r} is not "
            f"supported on the GPU path")
    qcode = _lib.PI0_QUANT_NONE
    if quant is not None:
        qcode = _lib.PI0_QUANT_Q3 if quant.quantize_dtype == "int3" else _lib.PI0_QUANT_Q4
    # attention logits operands (gemma_dual.py:115): fp32 (the reference's default) or the model
    # dtype; the reference would cast to any dtype, this build implements these two
    logits = getattr(cfg, "attn_logits_dtype", "float32")
    if logits == "float32":
        lcode = _lib.PI0_LOGITS_F32
    elif logits == dtype:
        lcode = _lib.PI0_LOGITS_MODEL_DTYPE
    else:
        raise ValueError(
            f"attn_logits_dtype={logits!r}: the B200 build computes the attention logits from "
            f"float32 or model-dtype ({dtype}) operands")
    return _lib.Pi0ConfigC(
        vlm_width=vlm.width, vlm_mlp_dim=vlm.mlp_dim, ae_width=ae.width, ae_mlp_dim=ae.mlp_dim,
        depth=vlm.depth, num_heads=vlm.num_heads, num_kv_heads=vlm.num_kv_heads,
        head_dim=vlm.head_dim, prefix_len=cfg.prefix_len, action_horizon=cfg.action_horizon,
        action_dim=cfg.action_dim, num_denoise_steps=cfg.num_denoise_steps,
        dtype=_lib.DTYPE_CODE[dtype], quant=qcode, max_batch=max_batch,
        rms_norm_eps=cfg.rms_norm_eps, rope_theta=cfg.rope_theta, attn_logits=lcode)


class Pi0Runtime:
    """Context of libpi0b200 on one GPU plus the VM-style function table."""

    def __init__(self, config: Pi0Config, device: Optional[int] = None, max_batch: int = 1,
                 quant=None):
        if not torch.cuda.is_available():
            raise RuntimeError("Pi0Runtime needs a CUDA GPU (sm_100a); this build has no CPU path")
        self.lib = _lib.load()
        self.config = config
        self.quant = quant
        self.dtype = quant.model_dtype if quant is not None else config.dtype
        self.device_index = torch.cuda.current_device() if device is None else int(device)
        self.device = torch.device("cuda", self.device_index)
        self.max_batch = int(max_batch)
        self._cfg = config_struct(config, max_batch, quant)
        self._ctx = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            rc = self.lib.pi0_create(ctypes.byref(self._cfg), self.device_index,
                                     ctypes.byref(self._ctx))
        if rc != 0:
            msg = self.lib.pi0_last_error(self._ctx).decode() if self._ctx else ""
            self.lib.pi0_destroy(self._ctx)
            self._ctx = None
            raise _lib.Pi0Error(rc, f"pi0_create: {msg}")
        self.named_params = backbone_named_params(config, quant=quant)
        lib_table = self.param_table()
        mine = [(n, tuple(p.shape), p.dtype) for n, p in self.named_params]
        if lib_table != mine:
            raise RuntimeError("libpi0b200 parameter table differs from mlc_vla's table")
        self._bound_key = None
        self._keep = None

    # -- lifetime --
    def close(self):
        if getattr(self, "_ctx", None):
            self.lib.pi0_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    # -- table --
    def param_table(self):
        out = []
        n = self.lib.pi0_num_params(self._ctx)
        name = ctypes.c_char_p()
        ndim = ctypes.c_int()
        shape = (ctypes.c_int64 * 2)()
        dt = ctypes.c_int()
        for i in range(n):
            _lib.check(self.lib.pi0_param_info(self._ctx, i, ctypes.byref(name), ctypes.byref(ndim),
                                               shape, ctypes.byref(dt)), self._ctx)
            out.append((name.value.decode(), tuple(int(shape[j]) for j in range(ndim.value)),
                        _lib.CODE_DTYPE[dt.value]))
        return out

    # -- parameters --
    def to_params(self, arrays: Sequence) -> List[torch.Tensor]:
        if len(arrays) != len(self.named_params):
            raise ValueError(f"expected {len(self.named_params)} arrays, got {len(arrays)}")
        out = []
        for a, (name, spec) in zip(arrays, self.named_params):
            t = to_device(a, spec.dtype, self.device)
            if tuple(t.shape) != tuple(spec.shape):
                raise ValueError(f"{name}: shape {tuple(t.shape)} != {tuple(spec.shape)}")
            out.append(t)
        return out

    def bind(self, params: Sequence) -> None:
        """Repack `params` into the library's weight arena unless they are already bound."""
        tensors = [p.torch if isinstance(p, DeviceArray) else p for p in params]
        key = tuple(t.data_ptr() for t in tensors)
        if key == self._bound_key:
            return
        if len(tensors) != len(self.named_params):
            raise ValueError(f"expected {len(self.named_params)} params, got {len(tensors)}")
        for t, (name, spec) in zip(tensors, self.named_params):
            if tuple(t.shape) != tuple(spec.shape) or t.dtype != TORCH_DTYPE[spec.dtype]:
                raise ValueError(f"{name}: expected {spec}, got {tuple(t.shape)} {t.dtype}")
            if not t.is_cuda or t.device.index != self.device_index or not t.is_contiguous():
                raise ValueError(f"{name}: must be a contiguous tensor on {self.device}")
        ptrs = (ctypes.c_void_p * len(tensors))(*key)
        _lib.check(self.lib.pi0_set_params(self._ctx, ptrs, len(tensors), self._stream()),
                   self._ctx, "pi0_set_params")
        self._bound_key = key
        self._keep = tensors

    # -- helpers --
    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _t(self, x, dtype):
        return to_device(x, dtype, self.device)

    def _batch_of(self, t: torch.Tensor, per_req: int) -> int:
        b = t.numel() // per_req
        if b * per_req != t.numel() or b < 1:
            raise ValueError(f"tensor of {t.numel()} elements is not a batch of {per_req}")
        if b > self.max_batch:
            raise ValueError(f"batch {b} exceeds max_batch {self.max_batch}")
        return b

    # -- exported functions (raw torch in/out) --
    def prefill(self, prefix_embs, prefix_mask, params=None, keys=None, values=None):
        if params is not None:
            self.bind(params)
        c = self.config
        vlm = c.vlm
        x = self._t(prefix_embs, self.dtype)
        b = self._batch_of(x, c.prefix_len * vlm.width)
        m = self._t(prefix_mask, "float32")
        if m.numel() == c.prefix_len and b > 1:
            m = m.reshape(1, -1).expand(b, -1).contiguous()
        if m.numel() != b * c.prefix_len:
            raise ValueError("prefix_mask must hold prefix_len values per request")
        shape = (vlm.depth, b, vlm.num_kv_heads, c.prefix_len, vlm.head_dim)
        if keys is None:
            keys = torch.empty(shape, dtype=torch.float32, device=self.device)
        if values is None:
            values = torch.empty(shape, dtype=TORCH_DTYPE[self.dtype], device=self.device)
        _lib.check(self.lib.pi0_prefill(self._ctx, b, x.data_ptr(), m.data_ptr(), keys.data_ptr(),
                                        values.data_ptr(), self._stream()), self._ctx,
                   "pi0_prefill")
        self._hold = (x, m)
        return keys, values

    def _suffix_args(self, keys, values, suffix_cos, suffix_sin, prefix_mask):
        c = self.config
        vlm = c.vlm
        k = self._t(keys, "float32")
        v = self._t(values, self.dtype)
        b = self._batch_of(k, vlm.depth * vlm.num_kv_heads * c.prefix_len * vlm.head_dim)
        half = vlm.head_dim // 2

        def per_req(x, n, dt):
            t = self._t(x, dt)
            if t.numel() == n and b > 1:
                t = t.reshape(1, -1).expand(b, -1).contiguous()
            if t.numel() != b * n:
                raise ValueError(f"expected {n} values per request, got {t.numel()} in total")
            return t

        sc = per_req(suffix_cos, c.suffix_len * half, "float32")
        ss = per_req(suffix_sin, c.suffix_len * half, "float32")
        m = per_req(prefix_mask, c.prefix_len, "float32")
        return b, k, v, sc, ss, m

    def denoise_step_kv(self, keys, values, x_t, time_emb, suffix_cos, suffix_sin, prefix_mask,
                        params=None, out=None):
        if params is not None:
            self.bind(params)
        c = self.config
        b, k, v, sc, ss, m = self._suffix_args(keys, values, suffix_cos, suffix_sin, prefix_mask)
        x = self._t(x_t, self.dtype)
        te = self._t(time_emb, self.dtype)
        if x.numel() != b * c.action_horizon * c.action_dim or te.numel() != c.action_expert.width:
            raise ValueError("x_t must be [B, S, D] and time_emb [1, W1]")
        if out is None:
            out = torch.empty((b, c.action_horizon, c.action_dim), dtype=torch.float32,
                              device=self.device)
        _lib.check(self.lib.pi0_denoise_step_kv(
            self._ctx, b, k.data_ptr(), v.data_ptr(), x.data_ptr(), te.data_ptr(), sc.data_ptr(),
            ss.data_ptr(), m.data_ptr(), out.data_ptr(), self._stream()), self._ctx,
            "pi0_denoise_step_kv")
        self._hold = (k, v, x, te, sc, ss, m)
        return out

    def denoise_step(self, prefix_embs, x_t, time_emb, params=None, out=None):
        """M0 joint step (``pi0_model.py:111-125``): prefix expert over the whole (all-valid)
        prefix and action expert over the suffix, v_t [B, S, D] fp32."""
        if params is not None:
            self.bind(params)
        c = self.config
        p = self._t(prefix_embs, self.dtype)
        b = self._batch_of(p, c.prefix_len * c.vlm.width)
        x = self._t(x_t, self.dtype)
        te = self._t(time_emb, self.dtype)
        if x.numel() != b * c.action_horizon * c.action_dim or te.numel() != c.action_expert.width:
            raise ValueError("x_t must be [B, S, D] and time_emb [1, W1]")
        if out is None:
            out = torch.empty((b, c.action_horizon, c.action_dim), dtype=torch.float32,
                              device=self.device)
        _lib.check(self.lib.pi0_denoise_step(self._ctx, b, p.data_ptr(), x.data_ptr(),
                                             te.data_ptr(), out.data_ptr(), self._stream()),
                   self._ctx, "pi0_denoise_step")
        self._hold = (p, x, te)
        return out

    def denoise_loop_kv(self, keys, values, x0, time_embs, suffix_cos, suffix_sin, prefix_mask,
                        params=None, out=None):
        if params is not None:
            self.bind(params)
        c = self.config
        b, k, v, sc, ss, m = self._suffix_args(keys, values, suffix_cos, suffix_sin, prefix_mask)
        x = self._t(x0, "float32")
        te = self._t(time_embs, self.dtype)
        if x.numel() != b * c.action_horizon * c.action_dim:
            raise ValueError("x0 must be [B, S, D]")
        if te.numel() != c.num_denoise_steps * c.action_expert.width:
            raise ValueError("time_embs must be [num_denoise_steps, W1]")
        if out is None:
            out = torch.empty((b, c.action_horizon, c.action_dim), dtype=torch.float32,
                              device=self.device)
        _lib.check(self.lib.pi0_denoise_loop_kv(
            self._ctx, b, k.data_ptr(), v.data_ptr(), x.data_ptr(), te.data_ptr(), sc.data_ptr(),
            ss.data_ptr(), m.data_ptr(), out.data_ptr(), self._stream()), self._ctx,
            "pi0_denoise_loop_kv")
        self._hold = (k, v, x, te, sc, ss, m)
        return out

    def linear(self, x: torch.Tensor, w: torch.Tensor, engine: int = 0) -> torch.Tensor:
        """y = x·wᵀ on the library's GEMM engine (0 auto, 1 tcgen05 tiles, 2 warp-level mma,
        3 weight-streaming split-K, 4 tcgen05 tiles split over K between a CTA pair, 5 tcgen05
        256×256 tiles on a CTA pair with cta_group::2 MMAs)."""
        x = self._t(x, self.dtype)
        w = self._t(w, self.dtype)
        m, k = x.shape
        n = w.shape[0]
        y = torch.empty((m, n), dtype=TORCH_DTYPE[self.dtype], device=self.device)
        _lib.check(self.lib.pi0_linear(self._ctx, x.data_ptr(), m, k, w.data_ptr(), n,
                                       y.data_ptr(), engine, self._stream()), self._ctx,
                   "pi0_linear")
        return y

    def device_error(self) -> int:
        return int(self.lib.pi0_device_error(self._ctx))

    # -- VM-style access --
    def __getitem__(self, name: str):
        if name == "prefill":
            def f(prefix_embs, prefix_mask, params):
                k, v = self.prefill(prefix_embs, prefix_mask, params)
                return (DeviceArray(k), DeviceArray(v))
        elif name == "denoise_step_kv":
            def f(keys, values, x_t, time_emb, suffix_cos, suffix_sin, prefix_mask, params):
                return DeviceArray(self.denoise_step_kv(keys, values, x_t, time_emb, suffix_cos,
                                                        suffix_sin, prefix_mask, params))
        elif name == "denoise_loop_kv":
            def f(keys, values, x0, time_embs, suffix_cos, suffix_sin, prefix_mask, params):
                return DeviceArray(self.denoise_loop_kv(keys, values, x0, time_embs, suffix_cos,
                                                        suffix_sin, prefix_mask, params))
        elif name == "denoise_step":
            def f(prefix_embs, x_t, time_emb, params):
                return DeviceArray(self.denoise_step(prefix_embs, x_t, time_emb, params))
        else:
            raise KeyError(f"{name!r} is not an exported function of this build "
                           f"(prefill, denoise_step_kv, denoise_loop_kv, denoise_step)")
        return f


def quantize_weight(w: torch.Tensor, preset) -> List[torch.Tensor]:
    """GPU group quantisation of one [out, in] weight (``GroupQuantize.quantize_weight``,
    ``quant.py:195-266``): returns [q_weight uint32 (as int32 storage), q_scale]."""
    lib = _lib.load()
    n, k = w.shape
    g, epw = preset.group_size, preset.num_elem_per_storage
    ng = -(-k // g)
    w = w.contiguous()
    qw = torch.empty((n, ng * (g // epw)), dtype=torch.int32, device=w.device)
    qs = torch.empty((n, ng), dtype=w.dtype, device=w.device)
    qcode = _lib.PI0_QUANT_Q3 if preset.quantize_dtype == "int3" else _lib.PI0_QUANT_Q4
    dcode = _lib.DTYPE_CODE[str(w.dtype).replace("torch.", "")]
    s = ctypes.c_void_p(torch.cuda.current_stream(w.device).cuda_stream)
    _lib.check(lib.pi0_quantize_weight(qcode, dcode, w.data_ptr(), n, k, qw.data_ptr(),
                                       qs.data_ptr(), s), None, "pi0_quantize_weight")
    return [qw, qs]


def dequantize_weight(q_weight: torch.Tensor, q_scale: torch.Tensor, preset, k: int) -> torch.Tensor:
    lib = _lib.load()
    n = q_weight.shape[0]
    w = torch.empty((n, k), dtype=q_scale.dtype, device=q_weight.device)
    qcode = _lib.PI0_QUANT_Q3 if preset.quantize_dtype == "int3" else _lib.PI0_QUANT_Q4
    dcode = _lib.DTYPE_CODE[str(q_scale.dtype).replace("torch.", "")]
    s = ctypes.c_void_p(torch.cuda.current_stream(q_weight.device).cuda_stream)
    _lib.check(lib.pi0_dequantize_weight(qcode, dcode, q_weight.contiguous().data_ptr(),
                                         q_scale.contiguous().data_ptr(), n, k, w.data_ptr(), s),
               None, "pi0_dequantize_weight")
    return w


def embed_language(table: torch.Tensor, input_ids, err: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``vm["embed_language"]`` (``pi0_model.py:101-104``): token ids [.., T] -> embeddings
    [.., T, width] = table[id] · sqrt(width) in the table's dtype (fp16 / bf16), on the table's
    device. Raises ValueError for an id outside the table unless `err` (a device int32 tensor)
    is given, in which case it is set to 1 and the row is zero. `out` (optional): a contiguous
    tensor of T·width elements to write into, e.g. the language rows of a prefix buffer."""
    lib = _lib.load()
    if table.dim() != 2 or not table.is_cuda:
        raise ValueError("table must be a [vocab, width] CUDA tensor")
    dev = table.device
    ids = torch.as_tensor(np.asarray(input_ids) if not isinstance(input_ids, torch.Tensor)
                          else input_ids).to(device=dev, dtype=torch.int32).contiguous()
    if out is None:
        out = torch.empty(tuple(ids.shape) + (table.shape[1],), dtype=table.dtype, device=dev)
    elif (out.numel() != ids.numel() * table.shape[1] or out.dtype != table.dtype
          or out.device != dev or not out.is_contiguous()):
        raise ValueError("out must be a contiguous tensor of n_tokens x width elements of the "
                         "table's dtype on its device")
    own = err is None
    flag = torch.zeros(1, dtype=torch.int32, device=dev) if own else err
    dcode = _lib.DTYPE_CODE[str(table.dtype).replace("torch.", "")]
    s = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(lib.pi0_embed_language(dcode, table.contiguous().data_ptr(), table.shape[0],
                                      table.shape[1], ids.data_ptr(), ids.numel(), out.data_ptr(),
                                      flag.data_ptr(), s), None, "pi0_embed_language")
    if own and int(flag.item()):
        raise ValueError("input_ids holds an id outside the embedding table")
    return out


__all__ = ["Pi0Runtime", "DeviceArray", "ParamSpec", "to_device", "quantize_weight",
           "dequantize_weight", "embed_language"]

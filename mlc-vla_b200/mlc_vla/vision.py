"""Python host for the vision stage of libpi0b200: ``vm["embed_image"]`` on the GPU.

The reference compiles the vision tower as its own engine (``Pi0Model(include={"vision"})``,
``python/mlc_vla/model/pi0/pi0_model.py:43-58,76-77``) and calls
``vm["embed_image"](image, params)`` (``pi0_model.py:97-99``, spec ``:212-215``): image
[1, 224, 224, 3] channels-last in the model dtype -> image tokens [1, 256, 2048]. ``VisionRuntime``
plays that engine's role; indexing it with ``"embed_image"`` gives a callable with the
reference's argument order (params last). Calls may also carry up to ``max_images`` images at once
(the three cameras of a π0.5 observation in one launch sequence).
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import torch

from . import _lib
from .model.pi0.pi0_config import Pi0Config
from .model.pi0.pi0_model import vision_named_params
from .runtime import TORCH_DTYPE, DeviceArray, to_device


def vision_config_struct(cfg: Pi0Config, max_images: int = 1) -> _lib.Pi0VisionConfigC:
    if cfg.dtype not in ("float16", "bfloat16"):
        raise ValueError(
            f"the B200 build computes in float16 or bfloat16; config.dtype={cfg.dtype!r} is not "
            f"supported on the GPU path")
    s = cfg.siglip
    return _lib.Pi0VisionConfigC(
        image_size=s.image_size, patch_size=s.patch_size, num_channels=s.num_channels,
        hidden_size=s.hidden_size, intermediate_size=s.intermediate_size,
        num_hidden_layers=s.num_hidden_layers, num_attention_heads=s.num_attention_heads,
        projection_dim=s.projection_dim, dtype=_lib.DTYPE_CODE[cfg.dtype],
        max_images=int(max_images), layer_norm_eps=s.layer_norm_eps)


class VisionRuntime:
    """A pi0_vision_ctx on one GPU (SigLIP So400m/14 + PaliGemma projector)."""

    def __init__(self, config: Pi0Config, device: Optional[int] = None, max_images: int = 1):
        if not torch.cuda.is_available():
            raise RuntimeError("VisionRuntime needs a CUDA GPU (sm_100a); this build has no CPU path")
        self.lib = _lib.load()
        self.config = config
        self.dtype = config.dtype
        self.device_index = torch.cuda.current_device() if device is None else int(device)
        self.device = torch.device("cuda", self.device_index)
        self.max_images = int(max_images)
        self._cfg = vision_config_struct(config, max_images)
        self._ctx = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            rc = self.lib.pi0_vision_create(ctypes.byref(self._cfg), self.device_index,
                                            ctypes.byref(self._ctx))
        if rc != 0:
            msg = self.lib.pi0_vision_last_error(self._ctx).decode() if self._ctx else ""
            self.lib.pi0_vision_destroy(self._ctx)
            self._ctx = None
            raise _lib.Pi0Error(rc, f"pi0_vision_create: {msg}")
        self.named_params = vision_named_params(config)
        mine = [(n, tuple(p.shape), p.dtype) for n, p in self.named_params]
        if self.param_table() != mine:
            raise RuntimeError("libpi0b200 vision parameter table differs from mlc_vla's table")
        self._bound_key = None
        self._keep = None

    def close(self):
        if getattr(self, "_ctx", None):
            self.lib.pi0_vision_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def _check(self, rc, what):
        _lib.check(rc, self._ctx, what, vision=True)

    def param_table(self):
        out = []
        name = ctypes.c_char_p()
        ndim = ctypes.c_int()
        shape = (ctypes.c_int64 * 2)()
        dt = ctypes.c_int()
        for i in range(self.lib.pi0_vision_num_params(self._ctx)):
            self._check(self.lib.pi0_vision_param_info(self._ctx, i, ctypes.byref(name),
                                                       ctypes.byref(ndim), shape, ctypes.byref(dt)),
                        "pi0_vision_param_info")
            out.append((name.value.decode(), tuple(int(shape[j]) for j in range(ndim.value)),
                        _lib.CODE_DTYPE[dt.value]))
        return out

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
        """Copy `params` into the library's weight arena unless they are already bound."""
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
        self._check(self.lib.pi0_vision_set_params(self._ctx, ptrs, len(tensors), self._stream()),
                    "pi0_vision_set_params")
        self._bound_key = key
        self._keep = tensors

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def embed_image(self, image, params=None, out=None) -> torch.Tensor:
        """image [n, S, S, C] (or [S, S, C]) -> image tokens [n, T, projection_dim] in the model
        dtype, T = (S / patch_size)²."""
        if params is not None:
            self.bind(params)
        s = self.config.siglip
        x = to_device(image, self.dtype, self.device)
        per = s.image_size * s.image_size * s.num_channels
        n = x.numel() // per
        if n < 1 or n * per != x.numel():
            raise ValueError(f"image of {x.numel()} elements is not a batch of "
                             f"[{s.image_size}, {s.image_size}, {s.num_channels}] images")
        if n > self.max_images:
            raise ValueError(f"{n} images exceed max_images {self.max_images}")
        shape = (n, s.num_patches, s.projection_dim)
        if out is None:
            out = torch.empty(shape, dtype=TORCH_DTYPE[self.dtype], device=self.device)
        elif tuple(out.shape) != shape or out.dtype != TORCH_DTYPE[self.dtype] or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous {shape} {self.dtype} tensor")
        self._check(self.lib.pi0_embed_image(self._ctx, n, x.data_ptr(), out.data_ptr(),
                                             self._stream()), "pi0_embed_image")
        return out

    def launch_count(self) -> int:
        return int(self.lib.pi0_vision_launch_count(self._ctx))

    def device_error(self) -> int:
        return int(self.lib.pi0_vision_device_error(self._ctx))

    def __getitem__(self, name: str):
        if name != "embed_image":
            raise KeyError(f"{name!r} is not an exported function of the vision engine (embed_image)")

        def f(image, params):
            return DeviceArray(self.embed_image(image, params))
        return f

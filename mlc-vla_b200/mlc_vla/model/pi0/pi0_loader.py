"""openpi π0 / π0.5 checkpoint (PyTorch ``PI0Pytorch`` state dict in safetensors) -> this
package's parameter names (``python/mlc_vla/model/pi0/pi0_loader.py`` in the reference).

The mapping has to be the reference's, key for key, for the same checkpoint to load into the
same parameters (``build_name_map``, reference ``pi0_loader.py:83-156``):

* both Gemma experts keep HF-style ``q/k/v/o_proj`` weights; expert 0 is PaliGemma's language
  model (``paligemma_with_expert.paligemma.model.language_model.``), expert 1 the action expert
  (``paligemma_with_expert.gemma_expert.model.``);
* ``gate_up_proj`` = rows of ``gate_proj`` followed by rows of ``up_proj`` (``:56-58``);
* plain RMSNorm scales are taken as stored (the model applies ``1 + scale``);
* π0.5 adaRMS norms of expert 1 (both per-layer norms and the final norm) take
  ``<norm>.dense.{weight,bias}`` as ``<norm>.1.modulation.{weight,bias}``;
* the SigLIP patch embedding conv ``[hidden, c, p, p]`` becomes a Linear ``[hidden, p·p·c]``
  in (p, p, c) order (``:61-65``);
* ``embed_tokens`` is the tied ``paligemma.lm_head.weight``;
* action in/out projections and the time MLP keep their names.

``load_params`` builds every mapped parameter, casts floating ones to the model dtype, and, given
the parameter table, asserts that nothing is missing and every shape matches (``:174-203``).
"""

from __future__ import annotations

from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from .pi0_config import Pi0Config

_ROOT = "paligemma_with_expert."
_PALIGEMMA = _ROOT + "paligemma.model."
_EXPERT_SRC = (_PALIGEMMA + "language_model.", _ROOT + "gemma_expert.model.")
_VISION = _PALIGEMMA + "vision_tower.vision_model."
_PROJECTOR = _PALIGEMMA + "multi_modal_projector.linear."
_TIED_EMBED = _ROOT + "paligemma.lm_head.weight"
_HEADS = ("action_in_proj", "action_out_proj", "time_mlp_in", "time_mlp_out")


class SourceSpec:
    """One target parameter: the source keys it is built from and the function that builds it
    (identity for a single key)."""

    def __init__(self, keys, fn: Optional[Callable[..., np.ndarray]] = None):
        self.keys: List[str] = [keys] if isinstance(keys, str) else list(keys)
        self.fn = fn

    def build(self, src: Dict[str, np.ndarray]) -> np.ndarray:
        arrays = [src[k] for k in self.keys]
        return self.fn(*arrays) if self.fn is not None else arrays[0]

    def __repr__(self):
        return f"SourceSpec({self.keys})"


def concat_gate_up(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """[F, W] gate and [F, W] up -> [2F, W] with the gate rows first."""
    return np.concatenate([gate, up], axis=0)


def conv_to_linear(conv: np.ndarray) -> np.ndarray:
    """Patch-embedding conv weight [hidden, c, p, p] -> Linear [hidden, p·p·c], (p, p, c) order."""
    hidden, c, p, q = conv.shape
    return np.ascontiguousarray(conv.transpose(0, 2, 3, 1)).reshape(hidden, p * q * c)


def _vision(config: Pi0Config) -> Iterable[Tuple[str, SourceSpec]]:
    yield "vision.patch_embedding.weight", SourceSpec(
        _VISION + "embeddings.patch_embedding.weight", conv_to_linear)
    yield "vision.patch_embedding.bias", SourceSpec(_VISION + "embeddings.patch_embedding.bias")
    yield "vision.position_embedding", SourceSpec(_VISION + "embeddings.position_embedding.weight")
    for i in range(config.siglip.num_hidden_layers):
        src, dst = f"{_VISION}encoder.layers.{i}.", f"vision.layers.{i}."
        for part in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                     "self_attn.out_proj", "mlp.fc1", "mlp.fc2", "layer_norm1", "layer_norm2"):
            for leaf in ("weight", "bias"):
                yield f"{dst}{part}.{leaf}", SourceSpec(f"{src}{part}.{leaf}")
    for leaf in ("weight", "bias"):
        yield f"vision.post_layernorm.{leaf}", SourceSpec(f"{_VISION}post_layernorm.{leaf}")
        yield f"vision.multi_modal_projector.{leaf}", SourceSpec(f"{_PROJECTOR}{leaf}")


def _backbone(config: Pi0Config) -> Iterable[Tuple[str, SourceSpec]]:
    adarms = (False, bool(config.pi05))
    for layer in range(config.vlm.depth):
        dst = f"backbone.layers.{layer}."
        for e, prefix in enumerate(_EXPERT_SRC):
            src = f"{prefix}layers.{layer}."
            for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
                yield (f"{dst}self_attn.experts.{e}.{proj}.weight",
                       SourceSpec(f"{src}self_attn.{proj}.weight"))
            yield (f"{dst}mlp.{e}.gate_up_proj.weight",
                   SourceSpec((f"{src}mlp.gate_proj.weight", f"{src}mlp.up_proj.weight"),
                              concat_gate_up))
            yield f"{dst}mlp.{e}.down_proj.weight", SourceSpec(f"{src}mlp.down_proj.weight")
            for norm in ("input_layernorm", "post_attention_layernorm"):
                if adarms[e]:
                    for leaf in ("weight", "bias"):
                        yield (f"{dst}{norm}.{e}.modulation.{leaf}",
                               SourceSpec(f"{src}{norm}.dense.{leaf}"))
                else:
                    yield f"{dst}{norm}.{e}.weight", SourceSpec(f"{src}{norm}.weight")
    for e, prefix in enumerate(_EXPERT_SRC):
        if adarms[e]:
            for leaf in ("weight", "bias"):
                yield (f"backbone.final_norm.{e}.modulation.{leaf}",
                       SourceSpec(f"{prefix}norm.dense.{leaf}"))
        else:
            yield f"backbone.final_norm.{e}.weight", SourceSpec(f"{prefix}norm.weight")


def build_name_map(config: Pi0Config) -> Dict[str, SourceSpec]:
    """Target parameter name -> SourceSpec, for every parameter the full model exports (vision
    tower, tied embedding, both experts, action heads, time MLP)."""
    name_map: Dict[str, SourceSpec] = dict(_vision(config))
    name_map["embed_tokens.weight"] = SourceSpec(_TIED_EMBED)
    name_map.update(_backbone(config))
    for head in _HEADS:
        for leaf in ("weight", "bias"):
            name_map[f"{head}.{leaf}"] = SourceSpec(f"{head}.{leaf}")
    return name_map


def load_safetensors(path: str, dtype: str = "float32") -> Dict[str, np.ndarray]:
    """An openpi PI0Pytorch safetensors file -> {key: numpy array}; 16-bit floats (bf16, fp16)
    are widened to `dtype`."""
    import torch
    from safetensors.torch import load_file

    out: Dict[str, np.ndarray] = {}
    for key, t in load_file(path).items():
        if t.dtype in (torch.bfloat16, torch.float16):
            t = t.to(torch.float32)
        out[key] = t.numpy().astype(np.dtype(dtype), copy=False)
    return out


def load_params(config: Pi0Config, src: Dict[str, np.ndarray], named_params=None,
                dtype: Optional[str] = None) -> Dict[str, np.ndarray]:
    """Build every mapped parameter from the source dict, floating ones cast to `dtype` (default
    the model dtype). With `named_params` ([(name, spec with .shape)], e.g. the runtime's
    table), every table entry must be built and have the table's shape; extra parameters (the
    vision tower when only the backbone is used) are allowed."""
    target = np.dtype(dtype or config.dtype) if (dtype or config.dtype) != "bfloat16" else np.float32
    params: Dict[str, np.ndarray] = {}
    for name, spec in build_name_map(config).items():
        if not all(k in src for k in spec.keys):
            if named_params is None or name in {n for n, _ in named_params}:
                missing = [k for k in spec.keys if k not in src]
                raise KeyError(f"{name}: source keys missing from the checkpoint: {missing}")
            continue
        arr = spec.build(src)
        if np.issubdtype(arr.dtype, np.floating):
            arr = arr.astype(target, copy=False)
        params[name] = arr
    if named_params is not None:
        missing = [n for n, _ in named_params if n not in params]
        if missing:
            raise KeyError(f"loader built no value for {len(missing)} parameters, e.g. {missing[:5]}")
        for n, spec in named_params:
            got, want = tuple(params[n].shape), tuple(int(s) for s in spec.shape)
            if got != want:
                raise ValueError(f"{n}: checkpoint gives shape {got}, the model expects {want}")
    return params


def to_openpi(config: Pi0Config, params: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """The inverse map, for the parameters present: {openpi key: array} (gate_up split back into
    gate and up rows; the patch-embedding Linear folded back into a conv)."""
    out: Dict[str, np.ndarray] = {}
    for name, spec in build_name_map(config).items():
        if name not in params:
            continue
        arr = params[name]
        if spec.fn is concat_gate_up:
            f = arr.shape[0] // 2
            out[spec.keys[0]], out[spec.keys[1]] = arr[:f], arr[f:]
        elif spec.fn is conv_to_linear:
            sig = config.siglip
            p, c = sig.patch_size, sig.num_channels
            out[spec.keys[0]] = np.ascontiguousarray(
                arr.reshape(arr.shape[0], p, p, c).transpose(0, 3, 1, 2))
        else:
            out[spec.keys[0]] = arr
    return out


def param_list(named_params: Sequence, params: Dict[str, np.ndarray]) -> List[np.ndarray]:
    """Arrays in parameter-table order (the list ``Pi0Runtime.to_params`` takes)."""
    return [params[n] for n, _ in named_params]


__all__ = ["SourceSpec", "build_name_map", "concat_gate_up", "conv_to_linear", "load_safetensors",
           "load_params", "to_openpi", "param_list"]

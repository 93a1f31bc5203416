"""Parameter table and exported-function specs of the π0.5 backbone build.

The reference builds ``Pi0Model(config, include={"backbone"})`` in TVM and takes its
``named_params`` from ``export_tvm`` (``python/mlc_vla/compile.py:24-38``,
``pi0_model.py:47-94``). Callers fill the packed parameter list **positionally** from that
table (``README.md:116-117``, ``tests/test_pizero_runner.py:31-38``), so this module
regenerates the same names, shapes, dtypes and order without TVM:

* module attribute order decides parameter order: ``backbone`` first
  (``pi0_model.py:81-82``), then ``action_in_proj``, ``action_out_proj``, ``time_mlp_in``,
  ``time_mlp_out`` (``pi0_model.py:84-88``);
* inside the backbone, every layer lists ``self_attn.experts.{0,1}.{q,k,v,o}_proj`` (no bias,
  ``gemma_dual.py:141-148``), then ``mlp.{0,1}.{gate_up,down}_proj`` (``gemma_dual.py:
  129-130,285``), then ``input_layernorm`` and ``post_attention_layernorm`` for both experts
  (``gemma_dual.py:286-291``); expert 0 uses a plain RMSNorm ``.weight`` and expert 1 (π0.5)
  an adaRMS ``.modulation.{weight,bias}`` of shape ``[3*width, width]``
  (``gemma_dual.py:63-73``); ``final_norm.{0,1}`` follows all layers (``gemma_dual.py:
  369-371``);
* ``model.to(config.dtype)`` casts every float parameter to the model dtype
  (``compile.py:33``), norm weights included.

For a group-quantised build every ``nn.Linear`` becomes ``q_weight`` (uint32), ``q_scale``
(model dtype) and, when the layer has one, ``bias`` (``quant.py:269-288``), in that order.
"""

from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional, Sequence, Tuple

from .pi0_config import Pi0Config

FUNCTIONS = ("prefill", "denoise_step_kv", "denoise_loop_kv", "denoise_step")


@dataclasses.dataclass(frozen=True)
class ParamSpec:
    """Shape and dtype of one packed parameter (the fields callers read from TVM params)."""

    shape: Tuple[int, ...]
    dtype: str

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n


@dataclasses.dataclass(frozen=True)
class LinearSpec:
    """One ``nn.Linear`` of the backbone: parameter name prefix, [out, in] and bias flag."""

    name: str
    out_features: int
    in_features: int
    bias: bool


def linear_layers(config: Pi0Config) -> List[LinearSpec]:
    """Every ``nn.Linear`` of the backbone build, in parameter-table order."""
    vlm, ae = config.vlm, config.action_expert
    hq = vlm.num_heads * vlm.head_dim
    hkv = vlm.num_kv_heads * vlm.head_dim
    experts = (vlm, ae)
    out: List[LinearSpec] = []
    for i in range(vlm.depth):
        p = f"backbone.layers.{i}."
        for e, c in enumerate(experts):
            a = f"{p}self_attn.experts.{e}."
            out.append(LinearSpec(a + "q_proj", hq, c.width, False))
            out.append(LinearSpec(a + "k_proj", hkv, c.width, False))
            out.append(LinearSpec(a + "v_proj", hkv, c.width, False))
            out.append(LinearSpec(a + "o_proj", c.width, hq, False))
        for e, c in enumerate(experts):
            out.append(LinearSpec(f"{p}mlp.{e}.gate_up_proj", 2 * c.mlp_dim, c.width, False))
            out.append(LinearSpec(f"{p}mlp.{e}.down_proj", c.width, c.mlp_dim, False))
        if config.pi05:
            for ln in ("input_layernorm", "post_attention_layernorm"):
                out.append(LinearSpec(f"{p}{ln}.1.modulation", 3 * ae.width, ae.width, True))
    if config.pi05:
        out.append(LinearSpec("backbone.final_norm.1.modulation", 3 * ae.width, ae.width, True))
    out.append(LinearSpec("action_in_proj", ae.width, config.action_dim, True))
    out.append(LinearSpec("action_out_proj", config.action_dim, ae.width, True))
    out.append(LinearSpec("time_mlp_in", ae.width, ae.width, True))
    out.append(LinearSpec("time_mlp_out", ae.width, ae.width, True))
    return out


def _linear_entries(lin: LinearSpec, dtype: str, quant=None) -> List[Tuple[str, ParamSpec]]:
    if quant is None:
        ent = [(lin.name + ".weight", ParamSpec((lin.out_features, lin.in_features), dtype))]
    else:
        ngroup = -(-lin.in_features // quant.group_size)
        ent = [
            (lin.name + ".q_weight",
             ParamSpec((lin.out_features, quant.num_storage_per_group * ngroup), quant.storage_dtype)),
            (lin.name + ".q_scale", ParamSpec((lin.out_features, ngroup), quant.model_dtype)),
        ]
    if lin.bias:
        ent.append((lin.name + ".bias", ParamSpec((lin.out_features,), dtype)))
    return ent


def backbone_named_params(config: Pi0Config, dtype: Optional[str] = None,
                          quant=None) -> List[Tuple[str, ParamSpec]]:
    """``[(name, ParamSpec)]`` in the reference's packed-parameter order.

    ``quant`` is a ``GroupQuantize`` preset (``mlc_vla.quant.PRESETS``) or ``None``.
    """
    dt = dtype or (quant.model_dtype if quant is not None else config.dtype)
    vlm, ae = config.vlm, config.action_expert
    lin = {l.name: l for l in linear_layers(config)}
    out: List[Tuple[str, ParamSpec]] = []

    def add_linear(name):
        out.extend(_linear_entries(lin[name], dt, quant))

    def add_norm(prefix: str, e: int, width: int):
        ada = config.pi05 and e == 1
        if ada:
            add_linear(f"{prefix}.{e}.modulation")
        else:
            out.append((f"{prefix}.{e}.weight", ParamSpec((width,), dt)))

    for i in range(vlm.depth):
        p = f"backbone.layers.{i}."
        for e in range(2):
            for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
                add_linear(f"{p}self_attn.experts.{e}.{proj}")
        for e in range(2):
            add_linear(f"{p}mlp.{e}.gate_up_proj")
            add_linear(f"{p}mlp.{e}.down_proj")
        for ln in ("input_layernorm", "post_attention_layernorm"):
            for e, c in enumerate((vlm, ae)):
                add_norm(p + ln, e, c.width)
    for e, c in enumerate((vlm, ae)):
        add_norm("backbone.final_norm", e, c.width)
    for name in ("action_in_proj", "action_out_proj", "time_mlp_in", "time_mlp_out"):
        add_linear(name)
    return out


def vision_named_params(config: Pi0Config, dtype: Optional[str] = None) -> List[Tuple[str, ParamSpec]]:
    """``[(name, ParamSpec)]`` of the vision stage (``Pi0Model(include={"vision"})``,
    ``pi0_model.py:76-77``) in the reference's creation order, ``siglip.py:92-102`` with
    ``SiglipEncoderLayer`` at ``:78-83``, ``SiglipAttention`` at ``:51-56`` and ``SiglipMLP`` at
    ``:40-42``: ``vision.patch_embedding.{weight,bias}`` ([hidden, p·p·c], the flattened-patch
    Linear), ``vision.position_embedding`` [num_patches, hidden], per layer
    ``self_attn.{q,k,v,out}_proj.{weight,bias}``, ``mlp.fc1``, ``mlp.fc2``, ``layer_norm1``,
    ``layer_norm2`` (``.weight``, ``.bias``), then ``post_layernorm`` and
    ``multi_modal_projector`` ([projection_dim, hidden]). Every entry in the model dtype."""
    dt = dtype or config.dtype
    s = config.siglip
    h, f = s.hidden_size, s.intermediate_size
    pdim = s.patch_size * s.patch_size * s.num_channels
    out: List[Tuple[str, ParamSpec]] = []

    def lin(name, o, i):
        out.append((name + ".weight", ParamSpec((o, i), dt)))
        out.append((name + ".bias", ParamSpec((o,), dt)))

    def norm(name, d):
        out.append((name + ".weight", ParamSpec((d,), dt)))
        out.append((name + ".bias", ParamSpec((d,), dt)))

    lin("vision.patch_embedding", h, pdim)
    out.append(("vision.position_embedding", ParamSpec((s.num_patches, h), dt)))
    for i in range(s.num_hidden_layers):
        p = f"vision.layers.{i}."
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            lin(p + "self_attn." + proj, h, h)
        lin(p + "mlp.fc1", f, h)
        lin(p + "mlp.fc2", h, f)
        norm(p + "layer_norm1", h)
        norm(p + "layer_norm2", h)
    norm("vision.post_layernorm", h)
    lin("vision.multi_modal_projector", s.projection_dim, h)
    return out


def function_specs(config: Pi0Config, batch: int = 1) -> Dict[str, List[Tuple[str, Tuple[int, ...], str]]]:
    """Argument names, shapes and dtypes of the exported functions.

    Mirrors ``Pi0Model.get_default_spec`` (``pi0_model.py:197-255``): the reference fixes the
    batch at 1; ``batch`` here extends every per-request tensor with a leading ``B`` (keys and
    values keep their layer axis first: ``[L, B, KV, P, hd]``).
    """
    vlm, ae = config.vlm, config.action_expert
    dt = config.dtype
    kv_shape = (vlm.depth, batch, vlm.num_kv_heads, config.prefix_len, vlm.head_dim)
    mask = (batch, 1, 1, config.prefix_len)
    rope = (batch, config.suffix_len, 1, vlm.head_dim // 2)
    act = (batch, config.action_horizon, config.action_dim)
    return {
        "prefill": [("prefix_embs", (batch, config.prefix_len, vlm.width), dt),
                    ("prefix_mask", mask, "float32")],
        "denoise_step_kv": [("keys", kv_shape, "float32"), ("values", kv_shape, dt),
                            ("x_t", act, dt), ("time_emb", (1, ae.width), dt),
                            ("suffix_cos", rope, "float32"), ("suffix_sin", rope, "float32"),
                            ("prefix_mask", mask, "float32")],
        "denoise_step": [("prefix_embs", (batch, config.prefix_len, vlm.width), dt),
                         ("x_t", act, dt), ("time_emb", (1, ae.width), dt)],
        "denoise_loop_kv": [("keys", kv_shape, "float32"), ("values", kv_shape, dt),
                            ("x0", act, "float32"),
                            ("time_embs", (config.num_denoise_steps, ae.width), dt),
                            ("suffix_cos", rope, "float32"), ("suffix_sin", rope, "float32"),
                            ("prefix_mask", mask, "float32")],
    }


class Pi0Model:
    """Backbone build of π0.5: exposes the parameter table and the function specs.

    Only the ``backbone`` stage (``pi0_model.py:47-59``) is on the hot path; building the
    vision or embedding stages raises ``NotImplementedError``.
    """

    def __init__(self, config: Pi0Config, include: Optional[Sequence[str]] = None):
        inc = {"backbone"} if include is None else set(include)
        if inc - {"backbone"}:
            raise NotImplementedError(
                f"stages {sorted(inc - {'backbone'})} are outside the M1 hot path of this build")
        self.config = config
        self.dtype = config.dtype

    def named_params(self, quant=None) -> List[Tuple[str, ParamSpec]]:
        return backbone_named_params(self.config, quant=quant)

    def get_default_spec(self, functions=None, batch: int = 1):
        spec = function_specs(self.config, batch)
        if functions is not None:
            spec = {k: spec[k] for k in functions}
        return spec

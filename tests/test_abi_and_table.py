"""CPU: the C-ABI library loads, exports every entry point declared in include/pi0b200.h, and
its parameter table equals the Python table (the reference's export order). No kernel runs."""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from tests.golden import recipes


def _header_functions():
    src = open(os.path.join(ROOT, "include", "pi0b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int64_t|int|const char\*)\s+(pi0_\w+)\s*\(", src, flags=re.M)))


def test_library_exports_every_header_symbol():
    from mlc_vla import _lib

    lib = _lib.load()
    names = _header_functions()
    assert len(names) >= 11
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.EXPORTED)


def _lib_table(cfg, quant=None, max_batch=1):
    from mlc_vla import _lib
    from mlc_vla.runtime import config_struct

    lib = _lib.load()
    c = config_struct(cfg, max_batch, quant)
    ctx = ctypes.c_void_p()
    rc = lib.pi0_create(ctypes.byref(c), 0, ctypes.byref(ctx))
    try:
        # without a GPU pi0_create reports a CUDA error, but the context (and its table) exist
        assert rc in (0, _lib.PI0_ERR_CUDA, _lib.PI0_ERR_UNSUPPORTED), lib.pi0_last_error(ctx)
        n = lib.pi0_num_params(ctx)
        out = []
        name, ndim, dt = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_int64 * 2)()
        for i in range(n):
            assert lib.pi0_param_info(ctx, i, ctypes.byref(name), ctypes.byref(ndim), shape,
                                      ctypes.byref(dt)) == 0
            out.append((name.value.decode(), tuple(shape[j] for j in range(ndim.value)),
                        _lib.CODE_DTYPE[dt.value]))
        return out
    finally:
        lib.pi0_destroy(ctx)


@pytest.mark.parametrize("kw", [recipes.MINI, recipes.DUMMY, recipes.FULL])
def test_library_table_matches_python_table(kw):
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    cfg = Pi0Config(**{**kw, "dtype": "float16"})
    mine = [(n, tuple(p.shape), p.dtype) for n, p in backbone_named_params(cfg)]
    assert _lib_table(cfg) == mine


@pytest.mark.parametrize("preset", ["q4f16_1", "q3f16_1", "q4bf16_1"])
def test_quantised_table_matches(preset):
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_model import backbone_named_params
    from mlc_vla.quant import PRESETS

    q = PRESETS[preset]
    cfg = Pi0Config(**{**recipes.FULL, "dtype": q.model_dtype})
    mine = [(n, tuple(p.shape), p.dtype) for n, p in backbone_named_params(cfg, quant=q)]
    assert _lib_table(cfg, quant=q) == mine


def test_full_table_order_and_sizes():
    """π0.5 backbone: 335 parameters, 2.412 B elements, modulation shapes [3072, 1024]."""
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_model import backbone_named_params

    npar = backbone_named_params(Pi0Config(dtype="float16"))
    assert len(npar) == 18 * 20 - 18 * 3 + 18 * 0 + 29 or len(npar) == 335
    assert sum(p.numel for _, p in npar) == 2_411_982_880
    names = [n for n, _ in npar]
    assert names[:4] == [f"backbone.layers.0.self_attn.experts.0.{x}_proj.weight" for x in "qkvo"]
    assert names[8:12] == ["backbone.layers.0.mlp.0.gate_up_proj.weight",
                           "backbone.layers.0.mlp.0.down_proj.weight",
                           "backbone.layers.0.mlp.1.gate_up_proj.weight",
                           "backbone.layers.0.mlp.1.down_proj.weight"]
    assert names[12:15] == ["backbone.layers.0.input_layernorm.0.weight",
                            "backbone.layers.0.input_layernorm.1.modulation.weight",
                            "backbone.layers.0.input_layernorm.1.modulation.bias"]
    assert names[-11:] == ["backbone.final_norm.0.weight", "backbone.final_norm.1.modulation.weight",
                           "backbone.final_norm.1.modulation.bias", "action_in_proj.weight",
                           "action_in_proj.bias", "action_out_proj.weight", "action_out_proj.bias",
                           "time_mlp_in.weight", "time_mlp_in.bias", "time_mlp_out.weight",
                           "time_mlp_out.bias"]
    shapes = dict(npar)
    assert shapes["backbone.layers.3.input_layernorm.1.modulation.weight"].shape == (3072, 1024)
    assert shapes["backbone.layers.3.mlp.0.gate_up_proj.weight"].shape == (32768, 2048)


def test_invalid_config_rejected_with_message():
    from mlc_vla import _lib

    lib = _lib.load()
    c = _lib.Pi0ConfigC(vlm_width=256, vlm_mlp_dim=1024, ae_width=128, ae_mlp_dim=512, depth=2,
                        num_heads=4, num_kv_heads=1, head_dim=48, prefix_len=64,
                        action_horizon=8, action_dim=8, num_denoise_steps=3, dtype=_lib.PI0_F16,
                        quant=0, max_batch=1, rms_norm_eps=1e-6, rope_theta=1e4)
    ctx = ctypes.c_void_p()
    rc = lib.pi0_create(ctypes.byref(c), 0, ctypes.byref(ctx))
    assert rc == _lib.PI0_ERR_UNSUPPORTED
    assert b"head_dim" in lib.pi0_last_error(ctx)
    lib.pi0_destroy(ctx)
    c.head_dim = 64
    c.dtype = _lib.PI0_F32
    rc = lib.pi0_create(ctypes.byref(c), 0, ctypes.byref(ctx))
    assert rc == _lib.PI0_ERR_UNSUPPORTED and b"float16" in lib.pi0_last_error(ctx)
    lib.pi0_destroy(ctx)


def test_cpu_targets_are_refused():
    from mlc_vla.compile import compile_model
    from mlc_vla.model.pi0 import Pi0Config

    with pytest.raises(ValueError, match="CUDA"):
        compile_model(Pi0Config(**{**recipes.MINI, "dtype": "float16"}), "c")


def test_embed_language_rejects_bad_arguments_before_any_device_work():
    """pi0_embed_language checks its arguments on the host (no GPU needed): null pointers,
    a width that is not a multiple of 8, and table / out pointers off a 16-byte boundary."""
    import ctypes

    from mlc_vla import _lib

    lib = _lib.load()
    vp = ctypes.c_void_p
    ok_ptr, bad_ptr = vp(0x100000), vp(0x100008)
    assert lib.pi0_embed_language(_lib.PI0_F16, None, 10, 64, ok_ptr, 1, ok_ptr, None, None) == 1
    assert lib.pi0_embed_language(_lib.PI0_F16, ok_ptr, 10, 60, ok_ptr, 1, ok_ptr, None, None) == 1
    assert lib.pi0_embed_language(_lib.PI0_F16, bad_ptr, 10, 64, ok_ptr, 1, ok_ptr, None, None) == 1
    assert lib.pi0_embed_language(_lib.PI0_F16, ok_ptr, 10, 64, ok_ptr, 1, bad_ptr, None, None) == 1
    assert lib.pi0_embed_language(_lib.PI0_F16, ok_ptr, 10, 64, ok_ptr, 0, ok_ptr, None, None) == 0


def _vision_table(cfg):
    from mlc_vla import _lib
    from mlc_vla.vision import vision_config_struct

    lib = _lib.load()
    c = vision_config_struct(cfg, 3)
    ctx = ctypes.c_void_p()
    rc = lib.pi0_vision_create(ctypes.byref(c), 0, ctypes.byref(ctx))
    try:
        assert rc in (0, _lib.PI0_ERR_CUDA), lib.pi0_vision_last_error(ctx)
        out = []
        name, ndim, dt = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_int64 * 2)()
        for i in range(lib.pi0_vision_num_params(ctx)):
            assert lib.pi0_vision_param_info(ctx, i, ctypes.byref(name), ctypes.byref(ndim),
                                             shape, ctypes.byref(dt)) == 0
            out.append((name.value.decode(), tuple(shape[j] for j in range(ndim.value)),
                        _lib.CODE_DTYPE[dt.value]))
        return out
    finally:
        lib.pi0_vision_destroy(ctx)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_vision_table_matches_python_table(dtype):
    """The vision engine's table (So400m: 439 entries) equals ``vision_named_params``, which is
    pinned to the reference loader's name map by test_siglip_oracle."""
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_model import vision_named_params
    from tests.golden import make_siglip_golden as G

    import dataclasses

    for cfg in (Pi0Config(dtype=dtype), G.configs()["mini"]):
        cfg = dataclasses.replace(cfg, dtype=dtype)
        mine = [(n, tuple(p.shape), p.dtype) for n, p in vision_named_params(cfg)]
        assert _vision_table(cfg) == mine


def test_invalid_vision_config_rejected_with_message():
    from mlc_vla import _lib

    lib = _lib.load()
    base = dict(image_size=224, patch_size=14, num_channels=3, hidden_size=1152,
                intermediate_size=4304, num_hidden_layers=27, num_attention_heads=16,
                projection_dim=2048, dtype=_lib.PI0_F16, max_images=3, layer_norm_eps=1e-6)
    for over, code, text in (({"dtype": _lib.PI0_F32}, _lib.PI0_ERR_UNSUPPORTED, b"float16"),
                             ({"image_size": 220}, _lib.PI0_ERR_INVALID, b"patch_size"),
                             ({"num_attention_heads": 6}, _lib.PI0_ERR_UNSUPPORTED, b"head_dim"),
                             ({"hidden_size": 4096, "num_attention_heads": 32},
                              _lib.PI0_ERR_UNSUPPORTED, b"2048"),
                             ({"max_images": 0}, _lib.PI0_ERR_INVALID, b"max_images")):
        c = _lib.Pi0VisionConfigC(**{**base, **over})
        ctx = ctypes.c_void_p()
        rc = lib.pi0_vision_create(ctypes.byref(c), 0, ctypes.byref(ctx))
        assert rc == code, (over, rc)
        assert text in lib.pi0_vision_last_error(ctx), (over, lib.pi0_vision_last_error(ctx))
        lib.pi0_vision_destroy(ctx)

"""Build and load ``libpi0b200.so`` (the sm_100a kernels behind include/pi0b200.h).

``build()`` compiles ``csrc/pi0_api.cu`` in-tree with nvcc for ``sm_100a``; ``load()`` opens the
library with ctypes and declares every entry point of the header. There is no fallback: when
the library is missing, ``load()`` raises.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
PROJECT_DIR = os.path.dirname(PKG_DIR)                      # mlc-vla_b200/
CSRC_DIR = os.path.join(PROJECT_DIR, "csrc")
INCLUDE_DIR = os.path.join(os.path.dirname(PROJECT_DIR), "include")
LIB_PATH = os.path.join(PKG_DIR, "lib", "libpi0b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]

PI0_OK, PI0_ERR_INVALID, PI0_ERR_CUDA, PI0_ERR_NO_PARAMS, PI0_ERR_DEVICE, PI0_ERR_UNSUPPORTED = range(6)
PI0_F16, PI0_BF16, PI0_F32, PI0_U32 = range(4)
PI0_QUANT_NONE, PI0_QUANT_Q4, PI0_QUANT_Q3 = range(3)
PI0_LOGITS_F32, PI0_LOGITS_MODEL_DTYPE = range(2)

DTYPE_CODE = {"float16": PI0_F16, "bfloat16": PI0_BF16, "float32": PI0_F32, "uint32": PI0_U32}
CODE_DTYPE = {v: k for k, v in DTYPE_CODE.items()}

EXPORTED = (
    "pi0_create", "pi0_destroy", "pi0_last_error", "pi0_num_params", "pi0_param_info",
    "pi0_set_params", "pi0_prefill", "pi0_denoise_step_kv", "pi0_denoise_loop_kv",
    "pi0_quantize_weight", "pi0_dequantize_weight", "pi0_launch_count", "pi0_profile_enable",
    "pi0_profile_read", "pi0_profile_families", "pi0_profile_family_name", "pi0_linear",
    "pi0_device_error", "pi0_div_check", "pi0_linear_noalloc", "pi0_wait_check",
    "pi0_embed_language", "pi0_denoise_step",
    "pi0_vision_create", "pi0_vision_destroy", "pi0_vision_last_error", "pi0_vision_num_params",
    "pi0_vision_param_info", "pi0_vision_set_params", "pi0_embed_image",
    "pi0_vision_launch_count", "pi0_vision_device_error", "pi0_vision_profile_enable",
    "pi0_vision_profile_read",
)


def _sources():
    return [os.path.join(CSRC_DIR, f) for f in sorted(os.listdir(CSRC_DIR))
            if f.endswith((".cu", ".cuh", ".h"))] + [os.path.join(INCLUDE_DIR, "pi0b200.h")]


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(s) > t for s in _sources())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libpi0b200.so for sm_100a (nvcc cross-compiles; no GPU needed)."""
    if not force and not needs_build():
        return LIB_PATH
    os.makedirs(os.path.dirname(LIB_PATH), exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = ["nvcc", *NVCC_FLAGS, f"-I{INCLUDE_DIR}", os.path.join(CSRC_DIR, "pi0_api.cu"), "-o", tmp]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=CSRC_DIR)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


class Pi0ConfigC(ctypes.Structure):
    """Mirror of ``struct pi0_config`` (include/pi0b200.h)."""

    _fields_ = [
        ("vlm_width", ctypes.c_int32), ("vlm_mlp_dim", ctypes.c_int32),
        ("ae_width", ctypes.c_int32), ("ae_mlp_dim", ctypes.c_int32),
        ("depth", ctypes.c_int32), ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("prefix_len", ctypes.c_int32), ("action_horizon", ctypes.c_int32),
        ("action_dim", ctypes.c_int32), ("num_denoise_steps", ctypes.c_int32),
        ("dtype", ctypes.c_int32), ("quant", ctypes.c_int32), ("max_batch", ctypes.c_int32),
        ("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
        ("attn_logits", ctypes.c_int32),
    ]


class Pi0VisionConfigC(ctypes.Structure):
    """Mirror of ``struct pi0_vision_config`` (include/pi0b200.h)."""

    _fields_ = [
        ("image_size", ctypes.c_int32), ("patch_size", ctypes.c_int32),
        ("num_channels", ctypes.c_int32), ("hidden_size", ctypes.c_int32),
        ("intermediate_size", ctypes.c_int32), ("num_hidden_layers", ctypes.c_int32),
        ("num_attention_heads", ctypes.c_int32), ("projection_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32), ("max_images", ctypes.c_int32),
        ("layer_norm_eps", ctypes.c_float),
    ]


_lib = None
_lock = threading.Lock()


def load():
    """Open libpi0b200.so and declare its C ABI. Raises if the library was not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -c 'import mlc_vla._lib as l; "
                f"l.build()'` (nvcc, sm_100a). This package has no CPU fallback.")
        lib = ctypes.CDLL(LIB_PATH)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        fp = ctypes.POINTER(ctypes.c_float)
        lib.pi0_create.argtypes = [ctypes.POINTER(Pi0ConfigC), i32, ctypes.POINTER(vp)]
        lib.pi0_destroy.argtypes = [vp]
        lib.pi0_last_error.argtypes = [vp]
        lib.pi0_last_error.restype = ctypes.c_char_p
        lib.pi0_num_params.argtypes = [vp]
        lib.pi0_param_info.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_char_p),
                                       ctypes.POINTER(i32), ctypes.POINTER(i64),
                                       ctypes.POINTER(i32)]
        lib.pi0_set_params.argtypes = [vp, ctypes.POINTER(vp), i32, vp]
        lib.pi0_prefill.argtypes = [vp, i32, vp, vp, vp, vp, vp]
        lib.pi0_denoise_step_kv.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp]
        lib.pi0_denoise_loop_kv.argtypes = [vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp]
        lib.pi0_quantize_weight.argtypes = [i32, i32, vp, i64, i64, vp, vp, vp]
        lib.pi0_dequantize_weight.argtypes = [i32, i32, vp, vp, i64, i64, vp, vp]
        lib.pi0_launch_count.argtypes = [vp]
        lib.pi0_launch_count.restype = ctypes.c_int64
        lib.pi0_profile_enable.argtypes = [vp, i32]
        lib.pi0_profile_read.argtypes = [vp, i32, ctypes.POINTER(i64),
                                         ctypes.POINTER(ctypes.c_double)]
        lib.pi0_profile_families.argtypes = []
        lib.pi0_profile_family_name.argtypes = [i32]
        lib.pi0_profile_family_name.restype = ctypes.c_char_p
        lib.pi0_linear.argtypes = [vp, vp, i32, i32, vp, i32, vp, i32, vp]
        lib.pi0_device_error.argtypes = [vp]
        lib.pi0_div_check.argtypes = [vp, vp, vp, i64, vp]
        lib.pi0_embed_language.argtypes = [i32, vp, i64, i32, vp, i32, vp, vp, vp]
        lib.pi0_denoise_step.argtypes = [vp, i32, vp, vp, vp, vp, vp]
        lib.pi0_wait_check.argtypes = [vp, i32, vp]
        lib.pi0_linear_noalloc.argtypes = [i32, vp, i32, i32, vp, i32, vp, vp]
        lib.pi0_vision_create.argtypes = [ctypes.POINTER(Pi0VisionConfigC), i32, ctypes.POINTER(vp)]
        lib.pi0_vision_destroy.argtypes = [vp]
        lib.pi0_vision_last_error.argtypes = [vp]
        lib.pi0_vision_last_error.restype = ctypes.c_char_p
        lib.pi0_vision_num_params.argtypes = [vp]
        lib.pi0_vision_param_info.argtypes = lib.pi0_param_info.argtypes
        lib.pi0_vision_set_params.argtypes = [vp, ctypes.POINTER(vp), i32, vp]
        lib.pi0_embed_image.argtypes = [vp, i32, vp, vp, vp]
        lib.pi0_vision_launch_count.argtypes = [vp]
        lib.pi0_vision_launch_count.restype = ctypes.c_int64
        lib.pi0_vision_device_error.argtypes = [vp]
        lib.pi0_vision_profile_enable.argtypes = [vp, i32]
        lib.pi0_vision_profile_read.argtypes = lib.pi0_profile_read.argtypes
        for name in EXPORTED:
            getattr(lib, name).restype = getattr(lib, name).restype or ctypes.c_int
        lib.pi0_last_error.restype = ctypes.c_char_p
        del fp
        _lib = lib
        return lib


class Pi0Error(RuntimeError):
    """A nonzero status from libpi0b200 (the analogue of TVM raising ``TVMError``)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"libpi0b200 error {code}: {msg}")
        self.code = code


def check(rc: int, ctx=None, what: str = "", vision: bool = False) -> None:
    """Raise Pi0Error for a nonzero status, with the context's last error text (`vision`: the
    context is a pi0_vision_ctx)."""
    if rc != PI0_OK:
        lib = load()
        err = lib.pi0_vision_last_error if vision else lib.pi0_last_error
        msg = err(ctx).decode() if ctx else ""
        raise Pi0Error(rc, f"{what}: {msg}" if what else msg)

"""Group weight quantisation presets (the reference's ``python/mlc_vla/quant.py``).

Same preset table as the reference (``quant.py:370-387``) and the same storage format: NK layout,
quantisation along K, ``q_weight`` [out, ceil(K/G)·G/epw] uint32 with element r of a word at bit
r·bits, ``q_scale`` [out, ceil(K/G)] in the model dtype, ``w = (code − max_int)·scale``.
``quantize_weight`` and ``dequantize`` run on the GPU (``pi0_quantize_weight`` /
``pi0_dequantize_weight`` in libpi0b200).
"""

from __future__ import annotations

import dataclasses
from typing import List

_BITS = {"int3": 3, "int4": 4, "int8": 8}


@dataclasses.dataclass
class GroupQuantize:
    name: str
    kind: str
    group_size: int
    quantize_dtype: str
    storage_dtype: str
    model_dtype: str
    linear_weight_layout: str
    quantize_embedding: bool = True
    quantize_final_fc: bool = True

    num_elem_per_storage: int = 0
    num_storage_per_group: int = 0
    max_int_value: int = 0

    def __post_init__(self):
        assert self.kind == "group-quant"
        bits = _BITS[self.quantize_dtype]
        storage_bits = 32 if self.storage_dtype == "uint32" else int(self.storage_dtype[4:])
        if storage_bits < bits:
            raise ValueError("Storage unit should be greater or equal to quantized element")
        self.num_elem_per_storage = storage_bits // bits
        if self.group_size % self.num_elem_per_storage != 0:
            raise ValueError("Group size should be divisible by numbers of elements per storage")
        self.num_storage_per_group = self.group_size // self.num_elem_per_storage
        self.max_int_value = (2 ** (bits - 1)) - 1
        self.linear_quant_axis = 0 if self.linear_weight_layout == "KN" else 1

    @property
    def bits(self) -> int:
        return _BITS[self.quantize_dtype]

    def quantize_weight(self, weight) -> List:
        """[out, in] model-dtype torch CUDA tensor -> [q_weight, q_scale] (GPU)."""
        from mlc_vla.runtime import quantize_weight

        if self.linear_weight_layout != "NK":
            raise NotImplementedError("only the NK layout of the presets is supported")
        return quantize_weight(weight, self)

    def dequantize(self, q_weight, q_scale, in_features: int):
        from mlc_vla.runtime import dequantize_weight

        return dequantize_weight(q_weight, q_scale, self, in_features)


PRESETS = {
    "q4bf16_1": GroupQuantize(name="q4bf16_1", kind="group-quant", group_size=32,
                              quantize_dtype="int4", storage_dtype="uint32",
                              model_dtype="bfloat16", linear_weight_layout="NK",
                              quantize_embedding=False, quantize_final_fc=True),
    "q4f16_1": GroupQuantize(name="q4f16_1", kind="group-quant", group_size=32,
                             quantize_dtype="int4", storage_dtype="uint32",
                             model_dtype="float16", linear_weight_layout="NK",
                             quantize_embedding=False, quantize_final_fc=True),
    "q3f16_1": GroupQuantize(name="q3f16_1", kind="group-quant", group_size=40,
                             quantize_dtype="int3", storage_dtype="uint32",
                             model_dtype="float16", linear_weight_layout="NK",
                             quantize_embedding=False, quantize_final_fc=True),
}


def get_quant(name: str) -> GroupQuantize:
    if name not in PRESETS:
        raise KeyError(f"unknown quantisation preset {name!r}; choose from {list(PRESETS)}")
    return PRESETS[name]

"""Runtime construction: the B200 build's counterpart of the reference's ``compile_model``.

The reference lowers the π0.5 backbone through TVM (``python/mlc_vla/compile.py:99-133``) and
returns ``(executable, named_params)``. Here there is nothing to compile at run time — the
kernels are prebuilt in ``libpi0b200.so`` — so ``compile_model`` creates a ``Pi0Runtime`` (the
library context on one GPU) and returns it with the same parameter table. Only the CUDA target
exists: asking for ``c`` / ``llvm`` raises instead of falling back to a CPU path.
"""

from __future__ import annotations

from typing import Optional

from mlc_vla.model.pi0 import Pi0Config
from mlc_vla.model.pi0.pi0_model import FUNCTIONS


def _check_target(target: str) -> None:
    kind = str(target).split()[0].split("-")[0]
    if kind != "cuda":
        raise ValueError(f"target {target!r}: the B200 build runs on CUDA (sm_100a) only; "
                         f"it has no CPU target")


def cublas_available() -> bool:
    """This build never dispatches to cuBLAS."""
    return False


def resolve_cublas(cublas, target_kind: str) -> bool:
    """Tri-state cuBLAS switch of the reference (``compile.py:55-76``); always False here."""
    return False


def compile_model(config: Pi0Config, target: str = "cuda", functions=None, cuda_graph: bool = False,
                  cublas=None, max_batch: int = 1, device: Optional[int] = None, quant=None):
    """Return ``(runtime, named_params)`` for the M1 functions of ``config``."""
    _check_target(target)
    fns = list(FUNCTIONS) if functions is None else list(functions)
    unknown = [f for f in fns if f not in FUNCTIONS]
    if unknown:
        raise NotImplementedError(f"functions {unknown} are outside the M1 hot path of this build")
    from mlc_vla.runtime import Pi0Runtime

    rt = Pi0Runtime(config, device=device, max_batch=max_batch, quant=quant)
    return rt, rt.named_params

"""Helpers shared by the GPU tests: runtimes on cuda:0 with seeded oracle weights."""

import numpy as np

from oracle import pi0_oracle as O
from tests.golden import recipes


def config(kw, dtype="float16", **over):
    from mlc_vla.model.pi0 import Pi0Config

    return Pi0Config(**{**kw, "dtype": dtype, **over})


class Model:
    """A runtime plus the same weights in the oracle's form."""

    def __init__(self, cfg, max_batch=1, seed=0):
        from mlc_vla.model.pi0.pi0_model import backbone_named_params
        from mlc_vla.runtime import Pi0Runtime

        self.cfg = cfg
        self.raw = O.random_params(backbone_named_params(cfg), seed=seed)
        self.p = O.prepare_params(self.raw, cfg.dtype)
        self.rt = Pi0Runtime(cfg, device=0, max_batch=max_batch)
        self.params = self.rt.to_params([self.raw[n] for n, _ in self.rt.named_params])
        self.rt.bind(self.params)

    def inputs(self, seed=1, batch=1):
        return recipes.inputs(self.cfg, seed=seed, batch=batch)

    def oracle_kv(self, prefix, pm):
        return O.prefill(self.p, self.cfg, prefix, pm)

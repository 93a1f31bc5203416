"""mlc_vla (B200 build): the π0.5 M1 inference hot path on hand-written sm_100a kernels.

Same import surface as the reference package for the M1 path: ``mlc_vla.model.pi0``
(``Pi0Config``), ``mlc_vla.sample`` (``PiZeroRunner``), ``mlc_vla.quant`` (group-quant
presets), ``mlc_vla.compile`` / ``mlc_vla.compile_quant`` (runtime construction).
"""

from .libinfo import __version__

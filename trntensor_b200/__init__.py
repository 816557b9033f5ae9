"""trntensor_b200 — B200-native DF-MP2 / AO→MO contraction path.

Drop-in for the trnsci/trntensor 0.4.0 public namespace
(trntensor/__init__.py:30-51): ``import trntensor_b200 as trntensor``.
``mp2_energy`` and ``ao_to_mo_transform`` run hand-written sm_100a kernels
(int8 Ozaki-split ``tcgen05.mma`` with exact int32 accumulation, for fp32
and for fp64) through the C ABI in ``include/trntensor_b200.h``;
``einsum``/``multi_einsum``/planning stay host Python. The tensor
decompositions are outside this build and raise ``NotImplementedError``.
"""

__version__ = "0.4.0+b200.1"

from .decompose import (
    cp_decompose,
    cp_reconstruct,
    tt_decompose,
    tt_reconstruct,
    tucker_decompose,
    tucker_reconstruct,
)
from .dispatch import HAS_NKI, from_xla, get_backend, set_backend, to_xla
from .einsum import einsum, multi_einsum
from .plan import (
    ContractionPlan,
    clear_plan_cache,
    estimate_flops,
    plan_cache_info,
    plan_contraction,
)
from .quantum import (
    ao_to_mo_transform,
    df_mp2_energy,
    mp2_energy,
    mp2_energy_dd,
    mp2_pair_energies,
)

__all__ = [
    "einsum",
    "multi_einsum",
    "ContractionPlan",
    "plan_contraction",
    "estimate_flops",
    "clear_plan_cache",
    "plan_cache_info",
    "cp_decompose",
    "cp_reconstruct",
    "tucker_decompose",
    "tucker_reconstruct",
    "tt_decompose",
    "tt_reconstruct",
    "HAS_NKI",
    "set_backend",
    "get_backend",
    "to_xla",
    "from_xla",
    "mp2_energy",
    "ao_to_mo_transform",
    "mp2_pair_energies",
    "mp2_energy_dd",
    "df_mp2_energy",
]

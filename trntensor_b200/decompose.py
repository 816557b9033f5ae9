"""Names of the reference's tensor decompositions (trntensor/decompose.py).

CP-ALS, Tucker/HOSVD and TT-SVD are iterative SVD/solve workloads outside
the DF-MP2 contraction path this package accelerates. The names exist so
that ``from trntensor_b200 import *`` matches the reference's namespace;
calling them raises ``NotImplementedError``.
"""

from __future__ import annotations


def _out_of_scope(name: str):
    def fn(*args, **kwargs):
        raise NotImplementedError(
            f"{name} is not part of trntensor_b200 (the B200 build covers the DF-MP2 "
            f"energy and AO->MO transform path); use trntensor.{name} from the reference package"
        )

    fn.__name__ = name
    fn.__doc__ = "Not available in trntensor_b200; raises NotImplementedError."
    return fn


cp_decompose = _out_of_scope("cp_decompose")
cp_reconstruct = _out_of_scope("cp_reconstruct")
tucker_decompose = _out_of_scope("tucker_decompose")
tucker_reconstruct = _out_of_scope("tucker_reconstruct")
tt_decompose = _out_of_scope("tt_decompose")
tt_reconstruct = _out_of_scope("tt_reconstruct")

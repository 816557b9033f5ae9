"""Import-compatibility shim for ``trntensor.nki.dispatch``.

Re-exports the names callers import from the reference's dispatch module
(trntensor/nki/dispatch.py: HAS_NKI, set_backend, get_backend, to_xla,
from_xla). The device wrappers live in :mod:`trntensor_b200.dispatch`.
"""

from ..dispatch import HAS_NKI, from_xla, get_backend, set_backend, to_xla

__all__ = ["HAS_NKI", "set_backend", "get_backend", "to_xla", "from_xla"]

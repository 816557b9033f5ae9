"""Import-compatibility shim for ``trntensor.nki`` (trntensor/nki/__init__.py).

``HAS_NKI`` is always False here; the executor is the sm_100a library.
"""

from ..dispatch import HAS_NKI, get_backend, set_backend

__all__ = ["HAS_NKI", "set_backend", "get_backend"]

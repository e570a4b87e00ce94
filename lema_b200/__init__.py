"""lema_b200 — B200-native (sm_100a) W8A8 streamed-layer hot path for LEMA.

The package holds the host side of the path: ctypes bindings of the C ABI
(``_native``), the torch-facing operators (``ops``), the ``nn.Linear``
drop-in (``modules``), the activation-checkpoint store and the native
transfer-engine shim (``_csrc._lema_cpp``).
"""
from ._native import LemaError, version  # noqa: F401

__all__ = ["LemaError", "version"]

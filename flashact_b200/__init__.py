"""B200-native (sm_100a) flow-matching action-expert denoise engine (pi0.5 / MolmoAct2 loop)."""
from ._capi import FlashActError, load_library  # noqa: F401
from .pi05 import Pi05ActionExpert  # noqa: F401
from .molmoact2 import MolmoAct2ActionExpert  # noqa: F401

__all__ = ["Pi05ActionExpert", "MolmoAct2ActionExpert", "FlashActError", "load_library"]

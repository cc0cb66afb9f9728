"""atomic_gdn2 (B200) -- Gated DeltaNet-2 operator on hand-written sm_100a kernels.

Drop-in for the reference package's public API (atomic_gdn2/__init__.py:1-10):
    BLRConfig, make_cfg, PROD, make_blr_trainable
"""
from .config import BLRConfig, make_cfg, PROD
from .pipeline import make_blr_trainable, set_checks, last_status

__version__ = "0.1.0"
__all__ = ["BLRConfig", "make_cfg", "PROD", "make_blr_trainable", "set_checks", "last_status"]

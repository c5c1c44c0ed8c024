"""qflash_b200 -- QFlash's integer-only attention forward on B200 (sm_100a).

Drop-in for the reference package's public surface (qflash/__init__.py):
``qflash`` (with ``qflash.forward``), ``QAttention``, ``QWindowAttention`` and
``patch_attention``.
"""
from .kernel import qflash
from .attention import QAttention, QWindowAttention, patch_attention

__all__ = ["qflash", "QAttention", "QWindowAttention", "patch_attention"]

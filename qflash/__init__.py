"""Import name of the reference package (``from qflash import qflash``),
served by qflash_b200's B200 implementation."""
from qflash_b200 import qflash, QAttention, QWindowAttention, patch_attention

__all__ = ["qflash", "QAttention", "QWindowAttention", "patch_attention"]
